// fqkv_prefill.cu -- the large-M (prefill) GEMM: out[M, N] = normed[M, H] * W[N, H]^T.
//
// Prefill is a dense contraction (arithmetic intensity 370-1170 FLOP/byte at the
// Llama-3-8B shape), so it is bound by the tensor cores.  The norm pre-pass
// (fqkv_norm.cu) has already written normed = dtype((h * rstd) * g) for every row; this
// kernel is a persistent, warp-specialised tcgen05 GEMM over 128 x BN output tiles:
//   warp 0     TMA producer: A tile (128 x 64) and B tile (BN x 64) per stage, both
//              K-major with 128-byte swizzle, into a STAGES-deep ring (no multicast).
//   warp 1     TMEM allocator and single-thread MMA issuer (tcgen05.mma kind::f16,
//              M = 128, N = BN, fp32 accumulators).  Two accumulator buffers in TMEM
//              let the epilogue of tile i overlap the main loop of tile i + 1.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, round to the working
//              dtype, store to global memory.
// Tiles are handed out round-robin (tile = blockIdx.x + i * gridDim.x), m fastest, so
// the CTAs running at the same time share weight tiles in L2.
// Every wait is bounded; a timeout sets the device status word and the CTA drains
// its loads and MMAs, frees TMEM and returns.
#include <cstdlib>
#include <type_traits>

#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

constexpr int kThreads = 192;
constexpr int kBM = 128;
constexpr int kKBlock = 64;
constexpr int kATileBytes = kBM * 128;

// Output staging of the CTA-pair kernel: two buffers of 128 rows x 64 columns (128 B
// rows, 128-byte swizzle), each stored by one TMA tensor store.
constexpr uint32_t kOutChunkBytes = kBM * 128;
constexpr uint32_t kOutStageBytes = 2 * kOutChunkBytes;

struct GLayout {
  uint32_t stage_bytes, stage_out, bars, tmem_slot, total;
};

__host__ __device__ inline GLayout make_glayout(int stages, int bn, uint32_t out_bytes = 0) {
  GLayout L;
  L.stage_bytes = kATileBytes + bn * 128;          // a multiple of 1024
  L.stage_out = stages * L.stage_bytes;            // output staging, 1024-aligned
  L.bars = L.stage_out + out_bytes;                // full[S], empty[S], tfull[2], tempty[2], done
  L.tmem_slot = L.bars + (2 * stages + 5) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Wait for this thread's TMEM loads.  The loaded registers pass through empty asm
// statements after the wait, so no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(a[i]), "+r"(b[i]));
}

template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmParams p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const GLayout L = make_glayout(stages, BN);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256u : 512u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.tiles_m * p.tiles_n;
  const int KB = p.kb_total;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(done_bar, 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      pdl_wait();  // A is written by the pre-pass
      const uint32_t tx = L.stage_bytes;
      bool ok = true;
      int s = 0, round = 0, issued = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mb = t % p.tiles_m, nb = t / p.tiles_m;
        for (int kb = 0; kb < KB; ++kb) {
          if (round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], tx);
          uint8_t* st = smem + s * L.stage_bytes;
          tma_load_2d(st, &tmA, &full[s], kb * kKBlock, mb * kBM);
          tma_load_2d(st + kATileBytes, &tmB, &full[s], kb * kKBlock, nb * BN);
          ++issued;
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
      }
      for (int j = max(0, issued - stages); j < issued; ++j) mbar_wait(&full[j % stages], (j / stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(kBM, BN, std::is_same<T, __nv_bfloat16>::value);
      bool ok = true;
      int s = 0, round = 0, li = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++li) {
        const int buf = li & 1, use = li >> 1;
        if (use > 0) ok = mbar_wait(&tempty[buf], (use - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < KB; ++kb) {
          ok = mbar_wait(&full[s], round & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * L.stage_bytes);
          const uint32_t b_base = a_base + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(d_tmem, make_sw128_desc(a_base + kk * 32), make_sw128_desc(b_base + kk * 32), idesc,
                     (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
        umma_commit(&tfull[buf]);
      }
      // Retire every MMA this thread issued before TMEM is freed (bounded).
      umma_commit(done_bar);
      mbar_wait(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    pdl_wait();  // out may still be read by the preceding grid
    const int q = warp & 3;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && ((p.ldo & 7) == 0);
    bool ok = true;
    int li = 0;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++li) {
      const int buf = li & 1, use = li >> 1;
      ok = mbar_wait(&tfull[buf], use & 1);
      if (!ok) break;
      tc_fence_after();
      const int mb = t % p.tiles_m, nb = t / p.tiles_m;
      const int64_t m = (int64_t)mb * kBM + q * 32 + lane;
      uint16_t* orow = p.out + m * p.ldo;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + c0, v);
        tmem_wait_ld();
        const int n0 = nb * BN + c0;
        const int cols = BN - c0 < 32 ? BN - c0 : 32;  // the last chunk of a tile may be narrower
        if (m < p.M) {
          uint32_t packed[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            packed[e] = (uint32_t)Elem<T>::from_f(__uint_as_float(v[2 * e])) |
                        ((uint32_t)Elem<T>::from_f(__uint_as_float(v[2 * e + 1])) << 16);
          if (vec_ok && cols == 32 && n0 + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(orow + n0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              dst[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
          } else {
            for (int e = 0; e < cols; ++e)
              if (n0 + e < p.N) orow[n0 + e] = (uint16_t)(packed[e >> 1] >> ((e & 1) * 16));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a 2-CTA cluster computes 256 x BN tiles.  CTA `rank`
// loads rows [256 mb + 128 rank, +128) of A and rows [BN nb + (BN/2) rank, +BN/2) of B
// into the same shared-memory offsets; the even CTA's MMA thread issues one
// tcgen05.mma.cta_group::2 per 16-wide K slice, reading both CTAs' halves, and D's rows
// [128 rank, +128) land in CTA `rank`'s TMEM.  Per SM that is half the B-operand traffic
// of a 128 x BN tile for the same FLOPs.  Barriers:
//   full[s]   (even CTA) both CTAs' loads of stage s, counted by TMA complete_tx;
//   empty[s]  (each CTA) stage s consumed: one commit multicast to both CTAs;
//   tfull[b]  (each CTA) accumulator b ready: one commit multicast to both CTAs;
//   tempty[b] (even CTA) accumulator b drained: one arrive per epilogue warp of both CTAs;
//   done      (each CTA) every MMA retired (multicast), before TMEM is freed.
// Epilogue: each CTA converts its 128 rows 64 columns at a time into a 128B-swizzled
// staging buffer (two, alternating) and one thread stores the 128 x 64 box with a TMA
// tensor store, when `out` allows a tensor map (p.out_tma); otherwise every thread
// stores its row.
template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, const GemmParams p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const GLayout L = make_glayout(stages, BN / 2, kOutStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256u : 512u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = p.tiles_m * p.tiles_n;  // tiles_m counts 256-row tiles
  const int KB = p.kb_total;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(done_bar, 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.out_tma) tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs have initialised their barriers and allocated TMEM
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t half_bytes = L.stage_bytes;
      // A static weight does not depend on the preceding grid: the weight halves of the
      // first ring round go out before the pre-pass (which writes A) has finished.
      int early = 0;
      if ((p.flags & FQKV_FLAG_STATIC_WEIGHTS) && pair < tiles) {
        const int nb0 = pair / p.tiles_m;
        early = min(stages, KB);
        for (int kb = 0; kb < early; ++kb) {
          if (rank == 0) mbar_arrive_expect_tx(&full[kb], 2 * half_bytes);
          tma_load_2d_pair(smem + kb * L.stage_bytes + kATileBytes, &tmB, mapa_shared(smem_u32(&full[kb]), 0),
                           kb * kKBlock, nb0 * BN + (int)rank * (BN / 2));
        }
      }
      pdl_wait();  // A is written by the pre-pass
      bool ok = true;
      int s = 0, round = 0, issued = 0;
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int mb = t % p.tiles_m, nb = t / p.tiles_m;
        for (int kb = 0; kb < KB; ++kb) {
          if (round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1);
          if (!ok) break;
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
          uint8_t* st = smem + s * L.stage_bytes;
          if (issued >= early) {
            // The even CTA's full[s] counts both CTAs' bytes.
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * half_bytes);
            tma_load_2d_pair(st + kATileBytes, &tmB, bar, kb * kKBlock, nb * BN + (int)rank * (BN / 2));
          }
          tma_load_2d_pair(st, &tmA, bar, kb * kKBlock, mb * 2 * kBM + (int)rank * kBM);
          ++issued;
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
      }
      // Every load of the pair completes on the even CTA's full barriers: that CTA waits for
      // the last `stages` of them (bounded), and both CTAs meet at the closing cluster
      // barrier, so neither leaves with a load of the pair in flight.
      if (rank == 0)
        for (int j = max(0, issued - stages); j < issued; ++j) mbar_wait<true>(&full[j % stages], (j / stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0) {
      if (rank == 0) {
        const uint32_t idesc = make_idesc_f16(2 * kBM, BN, std::is_same<T, __nv_bfloat16>::value);
        bool ok = true;
        int s = 0, round = 0, li = 0;
        for (int t = pair; t < tiles && ok; t += npairs, ++li) {
          const int buf = li & 1, use = li >> 1;
          if (use > 0) ok = mbar_wait<true>(&tempty[buf], (use - 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          for (int kb = 0; kb < KB; ++kb) {
            ok = mbar_wait<true>(&full[s], round & 1);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a_base = smem_u32(smem + s * L.stage_bytes);
            const uint32_t b_base = a_base + kATileBytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_pair(d_tmem, make_sw128_desc(a_base + kk * 32), make_sw128_desc(b_base + kk * 32), idesc,
                            (kb > 0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(&empty[s], 0x3);
            if (++s == stages) {
              s = 0;
              ++round;
            }
          }
          umma_commit_pair(&tfull[buf], 0x3);
        }
        umma_commit_pair(done_bar, 0x3);  // also on failure
      }
      mbar_wait<true>(done_bar, 0);  // every MMA retired before TMEM is freed
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    pdl_wait();  // out may still be read by the preceding grid
    const int q = warp & 3;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && ((p.ldo & 7) == 0);
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const int row = q * 32 + lane;  // this thread's row of the CTA's 128-row half
    uint8_t* const stage_out = smem + L.stage_out;
    const bool issuer = row == 0;  // issues and tracks this CTA's output TMA stores
    int n_out = 0;                 // output chunks staged so far (buffer n_out & 1 is next)
    bool ok = true;
    int li = 0;
    for (int t = pair; t < tiles && ok; t += npairs, ++li) {
      const int buf = li & 1, use = li >> 1;
      ok = mbar_wait<true>(&tfull[buf], use & 1);
      if (!ok) break;
      tc_fence_after();
      const int mb = t % p.tiles_m, nb = t / p.tiles_m;
      if (p.out_tma) {
        // TMEM -> registers (64 columns per wait) -> dtype -> staging buffer -> one TMA
        // store per 128 x 64 box.  Rows at or beyond M and columns at or beyond N lie
        // outside the tensor map and are not written.
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
        const int m0 = mb * 2 * kBM + (int)rank * kBM;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 64) {
          uint32_t va[32], vb[32];
          tmem_ld32(tbase + c0, va);
          tmem_ld32(tbase + c0 + 32, vb);
          tmem_wait_ld_regs(va, vb);
          if (c0 + 64 >= BN) {  // the accumulator is drained: the MMA may reuse it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty0 + buf * 8);
          }
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            pk[e] = Elem<T>::from_f2(__uint_as_float(va[2 * e]), __uint_as_float(va[2 * e + 1]));
            pk[16 + e] = Elem<T>::from_f2(__uint_as_float(vb[2 * e]), __uint_as_float(vb[2 * e + 1]));
          }
          uint8_t* sbuf = stage_out + (n_out & 1) * kOutChunkBytes;
          if (n_out >= 2) {  // the store issued from this buffer two chunks ago has read it
            if (issuer) bulk_wait_group_read<1>();
            asm volatile("bar.sync 2, 128;" ::: "memory");
          }
          // 16-byte chunk j of a 128-byte row sits at j ^ (row % 8): the 128-byte swizzle.
          uint8_t* srow = sbuf + row * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(srow + ((j ^ (row & 7)) << 4)) =
                make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          fence_proxy_async_smem();  // the staged tile is visible to the TMA unit
          asm volatile("bar.sync 2, 128;" ::: "memory");
          if (issuer && m0 < p.M && nb * BN + c0 < p.N) {
            tma_store_2d(&tmO, sbuf, nb * BN + c0, m0);
            bulk_commit_group();
          }
          ++n_out;
        }
        continue;
      }
      const int64_t m = (int64_t)mb * 2 * kBM + (int64_t)rank * kBM + row;
      uint16_t* orow = p.out + m * p.ldo;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + c0, v);
        tmem_wait_ld();
        const int n0 = nb * BN + c0;
        if (m < p.M) {
          uint32_t packed[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) packed[e] = Elem<T>::from_f2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
          if (vec_ok && n0 + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(orow + n0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              dst[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (n0 + e < p.N) orow[n0 + e] = (uint16_t)(packed[e >> 1] >> ((e & 1) * 16));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty0 + buf * 8);
    }
    if (issuer) bulk_wait_group<0>();  // every output store has completed
  }

  // ---------------------------------------------------------------- teardown
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA frees TMEM or leaves while the pair may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <typename T, int BN>
cudaError_t launch_pair_bn(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                           const GemmParams& p, bool pdl, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<T, BN>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), c.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3((unsigned)c.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmO, p, c.stages);
}

template <typename T, int BN>
cudaError_t launch_bn(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p,
                      bool pdl, cudaStream_t stream) {
  auto kern = gemm_kernel<T, BN>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), c.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)c.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = stream;
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, p, c.stages);
}

template <typename T>
cudaError_t launch_t(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                     const GemmParams& p, bool pdl, cudaStream_t stream) {
  if (c.pair) {
    switch (c.bn) {
      case 128: return launch_pair_bn<T, 128>(c, tmA, tmB, tmO, p, pdl, stream);
      case 256: return launch_pair_bn<T, 256>(c, tmA, tmB, tmO, p, pdl, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (c.bn) {
    case 128: return launch_bn<T, 128>(c, tmA, tmB, p, pdl, stream);
    case 192: return launch_bn<T, 192>(c, tmA, tmB, p, pdl, stream);
    case 256: return launch_bn<T, 256>(c, tmA, tmB, p, pdl, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

constexpr size_t kGemmSmemLimit = 232448;

// Kernel and tile width, from measurements on B200 at H = 4096, N = 6144 (graph-timed
// prefill, M = 512 ... 8192):
//   - CTA pairs with 256 x 256 tiles are the fastest kernel above 512 rows (M = 1024:
//     55 us against 57 us for the best single-CTA tile; M = 2048: 85 against 92 us);
//     at M <= 512 the single-CTA kernel fills more SMs and ties or wins.
//   - A 256 x 128 pair tile takes ~93% of the time of a 256 x 256 one, so pairs use
//     BN = 128 only when N <= 128.
//   - Single-CTA tiles: the fewest "tile-waves x (BN + 300)" (a wave of 128 x BN tiles
//     costs about BN + 300 in these units), ties going to the wider tile.
// FQKV_GEMM_PAIR=0 / 1 and FQKV_GEMM_BN override the choice (read once per process).
int gemm_pick_config(int M, int H, int N, int sm_count, GemmConfig* cfg) {
  (void)H;
  static const int force_bn = [] {
    const char* v = std::getenv("FQKV_GEMM_BN");
    return (v && *v) ? std::atoi(v) : 0;
  }();
  static const int force_pair = [] {  // -1: automatic
    const char* v = std::getenv("FQKV_GEMM_PAIR");
    return (v && *v) ? (std::atoi(v) != 0 ? 1 : 0) : -1;
  }();
  const bool pair = M > kBM && (force_pair >= 0 ? force_pair == 1 : M > 4 * kBM);
  const int units = pair ? sm_count / 2 : sm_count;  // concurrent tile workers
  const int bm = pair ? 2 * kBM : kBM;
  const int tiles_m = (M + bm - 1) / bm;
  int best_bn = 0;
  long best_cost = 0;
  for (int bn : {256, 192, 128}) {
    if (force_bn && bn != force_bn) continue;
    // 256 x 192 pair tiles (96 B rows per CTA) measured 2-3x slower than 256 x 256 on
    // B200, and their results are not covered by the tests: pairs use 256 or 128.
    if (pair && bn == 192) continue;
    if (pair && bn == 128 && N > 128 && !force_bn) continue;
    const long tiles = (long)tiles_m * ((N + bn - 1) / bn);
    const long waves = (tiles + units - 1) / units;
    const long cost = waves * (bn + 300);
    if (best_bn == 0 || cost < best_cost) {
      best_bn = bn;
      best_cost = cost;
    }
  }
  if (best_bn == 0) return FQKV_ERR_SCHEDULE;
  GemmConfig c{};
  c.bn = best_bn;
  c.pair = pair ? 1 : 0;
  const int b_rows = pair ? c.bn / 2 : c.bn;  // B rows each CTA loads per stage
  c.stages = 2;
  const uint32_t out_bytes = pair ? kOutStageBytes : 0;  // output staging of the pair kernel
  while (c.stages < 8 && 1024 + make_glayout(c.stages + 1, b_rows, out_bytes).total <= kGemmSmemLimit) ++c.stages;
  c.smem = 1024 + make_glayout(c.stages, b_rows, out_bytes).total;
  const long tiles = (long)tiles_m * ((N + c.bn - 1) / c.bn);
  c.grid = (int)(tiles < units ? tiles : units) * (pair ? 2 : 1);
  *cfg = c;
  return 0;
}

cudaError_t launch_gemm(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                        const GemmParams& p, bool bf16, bool pdl, cudaStream_t stream) {
  return bf16 ? launch_t<__nv_bfloat16>(c, tmA, tmB, tmO, p, pdl, stream)
              : launch_t<__half>(c, tmA, tmB, tmO, p, pdl, stream);
}

}  // namespace fqkv
