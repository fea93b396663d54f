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
#include <type_traits>

#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

constexpr int kThreads = 192;
constexpr int kBM = 128;
constexpr int kKBlock = 64;
constexpr int kATileBytes = kBM * 128;

struct GLayout {
  uint32_t stage_bytes, bars, tmem_slot, total;
};

__host__ __device__ inline GLayout make_glayout(int stages, int bn) {
  GLayout L;
  L.stage_bytes = kATileBytes + bn * 128;
  L.bars = stages * L.stage_bytes;                 // full[S], empty[S], tfull[2], tempty[2], done
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
        if (m < p.M) {
          uint32_t packed[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            packed[e] = (uint32_t)Elem<T>::from_f(__uint_as_float(v[2 * e])) |
                        ((uint32_t)Elem<T>::from_f(__uint_as_float(v[2 * e + 1])) << 16);
          if (vec_ok && n0 + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(orow + n0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              dst[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
          } else {
            for (int e = 0; e < 32; ++e)
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

template <typename T, int BN>
cudaError_t launch_bn(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p,
                      bool pdl, cudaStream_t stream) {
  auto kern = gemm_kernel<T, BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
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
cudaError_t launch_t(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p,
                     bool pdl, cudaStream_t stream) {
  switch (c.bn) {
    case 128: return launch_bn<T, 128>(c, tmA, tmB, p, pdl, stream);
    case 192: return launch_bn<T, 192>(c, tmA, tmB, p, pdl, stream);
    case 256: return launch_bn<T, 256>(c, tmA, tmB, p, pdl, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

constexpr size_t kGemmSmemLimit = 232448;

// Tile width BN: the candidate with the fewest "tile-waves x BN" (time proxy with one
// CTA per SM), ties going to the wider tile; ring depth as deep as shared memory allows.
int gemm_pick_config(int M, int H, int N, int sm_count, GemmConfig* cfg) {
  (void)H;
  const int tiles_m = (M + kBM - 1) / kBM;
  int best_bn = 0;
  long best_cost = 0;
  for (int bn : {256, 192, 128}) {
    const long tiles = (long)tiles_m * ((N + bn - 1) / bn);
    const long waves = (tiles + sm_count - 1) / sm_count;
    const long cost = waves * bn;
    if (best_bn == 0 || cost < best_cost) {
      best_bn = bn;
      best_cost = cost;
    }
  }
  GemmConfig c{};
  c.bn = best_bn;
  c.stages = 2;
  while (c.stages < 8 && 1024 + make_glayout(c.stages + 1, c.bn).total <= kGemmSmemLimit) ++c.stages;
  c.smem = 1024 + make_glayout(c.stages, c.bn).total;
  const long tiles = (long)tiles_m * ((N + c.bn - 1) / c.bn);
  c.grid = (int)(tiles < sm_count ? tiles : sm_count);
  *cfg = c;
  return 0;
}

cudaError_t launch_gemm(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p,
                        bool bf16, bool pdl, cudaStream_t stream) {
  return bf16 ? launch_t<__nv_bfloat16>(c, tmA, tmB, p, pdl, stream)
              : launch_t<__half>(c, tmA, tmB, p, pdl, stream);
}

}  // namespace fqkv
