// fqkv_streamk.cu -- small/mid-M GEMM after the norm pre-pass: swap-AB tcgen05 MMA with a
// stream-K split of the weight over every SM.
//
//   out[m, n] = sum_k normed[m, k] * W[n, k]     (normed written by norm_prepass_kernel)
//
// The weight is cut into T = ceil(N / 128) row tiles of KB = ceil(H / 64) k-blocks; the
// T * KB (tile, k-block) units are dealt to the G persistent CTAs (one per SM, no
// clusters) as G contiguous ranges whose lengths differ by at most one unit, so every
// SM streams the same number of weight bytes.  A range covers the end of one tile,
// whole tiles and/or the start of another; each such piece is a "segment".
//   warp 0     TMA producer: per unit, the 128 x 64 weight tile and the MPAD x 64 tile
//              of normalised rows (L2-resident) into one ring stage.
//   warp 1     TMEM allocator and single-thread MMA issuer: D^T[128 x MPAD] = W * normed^T
//              per segment in one of two TMEM accumulators (the epilogue of a segment
//              overlaps the next segment's MMAs).
//   warps 2-5  epilogue: a segment covering its whole tile is stored directly; a partial
//              segment writes its fp32 tile to this CTA's workspace slot, then counts
//              itself in the tile's arrival counter; the CTA that arrives last sums the
//              tile's slots in k order (so the result does not depend on arrival order)
//              and stores it.  Nobody waits for anybody: no spin on another CTA.
// Waits on this CTA's own mbarriers are bounded (fqkv_device.cuh).
#include <cstdlib>
#include <type_traits>

#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

constexpr int kThreads = 192;
constexpr int kTileRows = 128;
constexpr int kKBlock = 64;
constexpr int kWTileBytes = kTileRows * 128;

struct SLayout {
  uint32_t stage_bytes, bres, bars, flag, tmem_slot, total;
};

// b_slots > 0: the normalised rows of the CTA's k-blocks stay resident (b_slots tiles of
// MPAD x 64, loaded once); 0: each stage carries its own MPAD x 64 tile next to the weight.
__host__ __device__ inline SLayout make_slayout(int stages, int mpad, int b_slots) {
  SLayout L;
  L.stage_bytes = kWTileBytes + (b_slots > 0 ? 0 : mpad * 128);
  L.bres = stages * L.stage_bytes;
  L.bars = L.bres + b_slots * mpad * 128;  // full[S], empty[S], tfull[2], tempty[2], done, bfull
  L.flag = L.bars + (2 * stages + 6) * 8;
  L.tmem_slot = L.flag + 8;
  L.total = L.tmem_slot + 16;
  return L;
}

// First unit of CTA c when U units are dealt to G CTAs.
__host__ __device__ inline int64_t range_start(int64_t c, int64_t U, int64_t G) { return (c * U) / G; }

// CTA whose range contains unit u.
__device__ inline int owner_of(int64_t u, int64_t U, int64_t G) {
  int64_t c = (u * G) / U;
  while (c + 1 < G && range_start(c + 1, U, G) <= u) ++c;
  while (c > 0 && range_start(c, U, G) > u) --c;
  return (int)c;
}

template <typename T, int MPAD>
__global__ void __launch_bounds__(kThreads, 1)
    streamk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmB,
                   const StreamKParams p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SLayout L = make_slayout(stages, MPAD, p.b_slots);
  const bool bres = p.b_slots > 0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint64_t* bfull = tempty + 3;
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + L.flag);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  constexpr uint32_t kTmemCols = 2 * MPAD <= 32 ? 32u : 2 * MPAD <= 64 ? 64u : 2 * MPAD <= 128 ? 128u : 256u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.kb_total;
  const int64_t U = (int64_t)p.tiles * KB, G = gridDim.x;
  const int64_t u0 = range_start(blockIdx.x, U, G), u1 = range_start(blockIdx.x + 1, U, G);

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
    mbar_init(bfull, 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmB);
  }
  // k-blocks this CTA touches: a range of n_b (mod KB) starting at kb_s; the resident copy
  // of k-block kb lives in slot (kb - kb_s) mod KB.
  const int kb_s = (int)(u0 % KB);
  const int n_b = (int)((u1 - u0) < (int64_t)KB ? (u1 - u0) : (int64_t)KB);
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
      const uint32_t tx = L.stage_bytes;
      const int n_units = (int)(u1 - u0);
      const int pre = (p.flags & FQKV_FLAG_STATIC_WEIGHTS) ? min(stages, n_units) : 0;
      const bool hint = p.w_evict_first != 0;
      const uint64_t pol_w = policy_evict_first();
      auto load_w = [&](int slot, int64_t u) {
        void* dst = smem + slot * L.stage_bytes;
        const int kx = (int)(u % KB) * kKBlock, ky = (int)(u / KB) * kTileRows;
        if (hint) tma_load_2d_hint(dst, &tmW, &full[slot], kx, ky, pol_w);
        else tma_load_2d(dst, &tmW, &full[slot], kx, ky);
      };
      // The weight does not depend on the preceding grid when the caller says so: start
      // streaming it before the pre-pass has finished.
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], tx);
        load_w(i, u0 + i);
      }
      pdl_wait();  // normalised rows come from the pre-pass
      if (bres) {
        mbar_arrive_expect_tx(bfull, (uint32_t)(n_b * MPAD * 128));
        for (int j = 0; j < n_b; ++j)
          tma_load_2d(smem + L.bres + j * (MPAD * 128), &tmB, bfull, ((kb_s + j) % KB) * kKBlock, 0);
      } else {
        for (int i = 0; i < pre; ++i)
          tma_load_2d(smem + i * L.stage_bytes + kWTileBytes, &tmB, &full[i], (int)((u0 + i) % KB) * kKBlock, 0);
      }
      bool ok = true;
      int s = pre % stages, round = pre / stages, issued = pre;
      for (int64_t u = u0 + pre; u < u1; ++u) {
        if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1))) break;
        mbar_arrive_expect_tx(&full[s], tx);
        load_w(s, u);
        if (!bres) tma_load_2d(smem + s * L.stage_bytes + kWTileBytes, &tmB, &full[s], (int)(u % KB) * kKBlock, 0);
        ++issued;
        if (++s == stages) {
          s = 0;
          ++round;
        }
      }
      for (int j = max(0, issued - stages); j < issued; ++j) mbar_wait(&full[j % stages], (j / stages) & 1);
      if (bres) mbar_wait(bfull, 0);
      (void)ok;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(kTileRows, MPAD, std::is_same<T, __nv_bfloat16>::value);
      bool ok = !bres || mbar_wait(bfull, 0);
      int s = 0, round = 0, seg = 0;
      bool first = true;
      uint32_t d_tmem = tmem_base;
      for (int64_t u = u0; u < u1 && ok; ++u) {
        const int kb = (int)(u % KB);
        if (u == u0 || kb == 0) {  // a segment starts
          const int buf = seg & 1, use = seg >> 1;
          if (use > 0 && !(ok = mbar_wait(&tempty[buf], (use - 1) & 1))) break;
          tc_fence_after();
          d_tmem = tmem_base + buf * MPAD;
          first = true;
        }
        if (!(ok = mbar_wait(&full[s], round & 1))) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + s * L.stage_bytes);
        const uint32_t b_base =
            bres ? smem_u32(smem + L.bres + (((kb - kb_s + KB) % KB) * (MPAD * 128))) : a_base + kWTileBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(d_tmem, make_sw128_desc(a_base + kk * 32), make_sw128_desc(b_base + kk * 32), idesc,
                   (first && kk == 0) ? 0u : 1u);
        first = false;
        umma_commit(&empty[s]);
        if (++s == stages) {
          s = 0;
          ++round;
        }
        if (kb == KB - 1 || u == u1 - 1) {  // the segment ends
          umma_commit(&tfull[seg & 1]);
          ++seg;
        }
      }
      umma_commit(done_bar);
      mbar_wait(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;  // weight row within the tile = output feature
    pdl_wait();
    int seg = 0;
    for (int64_t u = u0; u < u1;) {
      const int t = (int)(u / KB);
      const int kb_a = (int)(u % KB);
      const int64_t u_end = min(u1, (int64_t)(t + 1) * KB);  // exclusive
      const bool whole = kb_a == 0 && u_end == (int64_t)(t + 1) * KB;
      const int buf = seg & 1;
      // All 128 epilogue threads take the same branch (they meet at named barriers below).
      if (!bar_and(1, 128, mbar_wait(&tfull[buf], (seg >> 1) & 1))) break;
      tc_fence_after();
      const int n = t * kTileRows + row;
      float* slot = nullptr;
      if (!whole) {
        // Only a CTA's first and last segments can be partial: the first goes to slot 0,
        // the last (if different) to slot 1.
        const int jj = (u == u0) ? 0 : 1;
        slot = p.partials + ((int64_t)blockIdx.x * 2 + jj) * (MPAD * kTileRows);
      }
#pragma unroll
      for (int c0 = 0; c0 < MPAD; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + buf * MPAD + c0, v);
        tmem_wait_ld();
        if (c0 < p.M) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (c0 + e >= p.M) break;
            if (whole) {
              if (n < p.N) p.out[(int64_t)(c0 + e) * p.ldo + n] = Elem<T>::from_f(__uint_as_float(v[e]));
            } else {
              slot[(c0 + e) * kTileRows + row] = __uint_as_float(v[e]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      if (!whole) {
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int c_first = owner_of((int64_t)t * KB, U, G);
        const int c_last = owner_of((int64_t)(t + 1) * KB - 1, U, G);
        if (et == 0) {
          const int old = atomicAdd(&p.counters[t], 1);
          *last_flag = (old == c_last - c_first) ? 1 : 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          __threadfence();
          // Sum the tile's partial slots in k order: CTA c_first's piece (its last segment
          // unless its range starts exactly at this tile), then every later CTA's first.
          // Rows go 16 at a time with all loads of a slot issued together.
          const bool first_starts_here = range_start(c_first, U, G) == (int64_t)t * KB;
          for (int m0 = 0; m0 < p.M; m0 += 16) {
            float acc[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
              const int jj = (c == c_first && !first_starts_here) ? 1 : 0;
              const float* src = p.partials + ((int64_t)c * 2 + jj) * (MPAD * kTileRows) + m0 * kTileRows + row;
              float v[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = (m0 + e < p.M) ? __ldcg(src + e * kTileRows) : 0.f;
#pragma unroll
              for (int e = 0; e < 16; ++e) acc[e] += v[e];
            }
            if (n < p.N) {
#pragma unroll
              for (int e = 0; e < 16; ++e)
                if (m0 + e < p.M) p.out[(int64_t)(m0 + e) * p.ldo + n] = Elem<T>::from_f(acc[e]);
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      ++seg;
      u = u_end;
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

template <typename T, int MPAD>
cudaError_t launch_t(const StreamKConfig& c, const CUtensorMap& tmW, const CUtensorMap& tmB,
                     const StreamKParams& p, bool pdl, cudaStream_t stream) {
  auto kern = streamk_kernel<T, MPAD>;
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
  return cudaLaunchKernelEx(&cfg, kern, tmW, tmB, p, c.stages);
}

template <typename T>
cudaError_t launch_dt(const StreamKConfig& c, const CUtensorMap& tmW, const CUtensorMap& tmB,
                      const StreamKParams& p, bool pdl, cudaStream_t stream) {
  switch (c.mpad) {
    case 16: return launch_t<T, 16>(c, tmW, tmB, p, pdl, stream);
    case 32: return launch_t<T, 32>(c, tmW, tmB, p, pdl, stream);
    case 64: return launch_t<T, 64>(c, tmW, tmB, p, pdl, stream);
    case 128: return launch_t<T, 128>(c, tmW, tmB, p, pdl, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

constexpr size_t kSmemLimitSK = 232448;

int streamk_mpad(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// Workspace after the normalised rows: per-CTA partial slots, then one arrival counter
// per weight tile.  Sized for kStreamKMaxGrid CTAs so it is known without a device.
int64_t streamk_partials_bytes(int M) { return (int64_t)kStreamKMaxGrid * 2 * streamk_mpad(M) * kTileRows * 4; }
int64_t streamk_counters_bytes(int N) { return (int64_t)((N + kTileRows - 1) / kTileRows) * 4; }

static int env_or(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

// Grid: every SM (FQKV_SPLIT_CTAS_PER_SM CTAs each, default 1), at most one CTA per unit.
// The normalised rows stay resident when the CTA's k-blocks fit in kBResidentMax bytes.
// Ring: as deep as fits in the per-CTA share of shared memory (FQKV_SPLIT_STAGES overrides).
int streamk_pick_config(int M, int H, int N, int sm_count, StreamKConfig* cfg) {
  StreamKConfig c{};
  c.mpad = streamk_mpad(M);
  if (M > 128) return FQKV_ERR_SCHEDULE;
  const int KB = (H + kKBlock - 1) / kKBlock;
  const int64_t units = (int64_t)((N + kTileRows - 1) / kTileRows) * KB;
  const int per_sm = max(1, min(2, env_or("FQKV_SPLIT_CTAS_PER_SM", 1)));
  int64_t g = (int64_t)sm_count * per_sm;
  if (g > kStreamKMaxGrid) g = kStreamKMaxGrid;
  if (units < g) g = units;
  c.grid = (int)g;
  const int64_t max_units = (units + g - 1) / g;
  const int b_slots = (int)(max_units < (int64_t)KB ? max_units : (int64_t)KB);
  const int bres_max = env_or("FQKV_SPLIT_BRES_MAX", 48 * 1024);
  c.b_slots = (int64_t)b_slots * c.mpad * 128 <= bres_max ? b_slots : 0;
  const size_t limit = kSmemLimitSK / per_sm - 1024;
  c.stages = 2;
  while (c.stages < 16 && 1024 + make_slayout(c.stages + 1, c.mpad, c.b_slots).total <= limit) ++c.stages;
  c.stages = env_or("FQKV_SPLIT_STAGES", c.stages);
  c.w_evict_first = env_or("FQKV_W_EVICT_FIRST", 1);
  if (c.stages < 2 || 1024 + make_slayout(c.stages, c.mpad, c.b_slots).total > kSmemLimitSK) return FQKV_ERR_SCHEDULE;
  c.smem = 1024 + make_slayout(c.stages, c.mpad, c.b_slots).total;
  *cfg = c;
  return 0;
}

cudaError_t launch_streamk(const StreamKConfig& c, const CUtensorMap& tmW, const CUtensorMap& tmB,
                           const StreamKParams& p, bool bf16, bool pdl, cudaStream_t stream) {
  return bf16 ? launch_dt<__nv_bfloat16>(c, tmW, tmB, p, pdl, stream)
              : launch_dt<__half>(c, tmW, tmB, p, pdl, stream);
}

}  // namespace fqkv
