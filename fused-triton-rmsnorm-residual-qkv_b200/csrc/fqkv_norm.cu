// fqkv_norm.cu -- the two CUDA-core kernels of the library:
//
//  * norm_prepass_kernel: residual add + RMSNorm of whole rows.  Writes the updated
//    residual (bit-exact x + r in the working dtype, baseline.py:48) and the
//    normalised activations dtype((h * rstd) * g) (baseline.py:59-62) to a scratch
//    matrix that the tensor-core GEMMs read with TMA.  One CTA per row.
//
//  * simt_kernel: the generic fused op for shapes/strides the TMA paths cannot take
//    (H not a multiple of 8, unaligned pointers).  Same two-phase structure as the
//    reference's 2-D-grid Triton kernel (kernel.py:122-215): phase 1 is the row
//    variance over all of H, phase 2 re-reads the rows, normalises and accumulates
//    against the weight tile in fp32.
#include "fqkv_kernels.cuh"

namespace fqkv {

// ---------------------------------------------------------------------------
// Pre-pass: one CTA (256 threads) per row; requires H % 8 == 0, H <= 16384 and
// 16-byte aligned rows.  Each thread keeps CPT chunks of 8 elements in registers
// (CPT = ceil(H / 2048), so the register footprint, and hence occupancy, follows H).
// ---------------------------------------------------------------------------
template <typename T, int CPT>
__global__ void __launch_bounds__(256, CPT <= 2 ? 4 : 1) norm_prepass_kernel(const PrepassParams p) {
  constexpr int kMaxChunks = CPT;
  __shared__ float warp_sums[8];
  pdl_launch_dependents();
  pdl_wait();

  const int64_t m = blockIdx.x;
  const int tid = threadIdx.x;
  const int nchunks = (int)(p.H / 8);
  if (p.counters && blockIdx.x == 0)
    for (int i = tid; i < p.n_counters; i += 256) p.counters[i] = 0;
  const uint16_t* xrow = p.x + m * p.ldx;
  const uint16_t* rrow = p.r ? p.r + m * p.ldr : nullptr;

  // Issue every load of the row (x, residual and the gain) before using any of them, so
  // the row costs one memory latency.
  uint4 h[kMaxChunks], rv[kMaxChunks];
  float4 g[kMaxChunks][2];
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = tid + i * 256;
    if (c < nchunks) {
      h[i] = __ldg(reinterpret_cast<const uint4*>(xrow + (int64_t)c * 8));
      if (rrow) rv[i] = __ldg(reinterpret_cast<const uint4*>(rrow + (int64_t)c * 8));
      load_gain8(p.g, p.gdt, (int64_t)c * 8, g[i]);
    }
  }
  uint64_t ss2 = 0ull;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = tid + i * 256;
    if (c < nchunks) {
      if (rrow) h[i] = add8_rn<T>(h[i], rv[i]);
      ss2 = sumsq8_f2<T>(h[i], ss2);
      if (p.rout) *reinterpret_cast<uint4*>(p.rout + m * p.ldro + (int64_t)c * 8) = h[i];
    }
  }
  float lo, hi;
  f2_unpack(ss2, lo, hi);
  float ss = lo + hi;
  // Block reduction in a fixed order (deterministic).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) warp_sums[tid >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) total += warp_sums[w];
  const float rstd = row_rstd(total, p.H, p.eps);
  const uint64_t rs2 = f2_pack(rstd, rstd);

  uint16_t* nrow = p.normed + m * p.H;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = tid + i * 256;
    if (c < nchunks) {
      const uint64_t g2[4] = {f2_pack(g[i][0].x, g[i][0].y), f2_pack(g[i][0].z, g[i][0].w),
                              f2_pack(g[i][1].x, g[i][1].y), f2_pack(g[i][1].z, g[i][1].w)};
      *reinterpret_cast<uint4*>(nrow + (int64_t)c * 8) = normalize8_f2<T>(h[i], rs2, g2);
    }
  }
}

// ---------------------------------------------------------------------------
// Generic SIMT kernel.  Tile: 8 token rows x 64 output features, K step 64.
// grid = (ceil(N / 64), ceil(M / 8)), 256 threads.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) simt_kernel(const SimtParams p) {
  constexpr int BM = 8, BN = 64, BK = 64;
  __shared__ float rstd_s[BM];
  __shared__ float nrm[BM][BK];
  __shared__ float wt[BN][BK + 1];
  pdl_launch_dependents();
  pdl_wait();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  // Phase 1: one warp per row -- sum of squares of h = dtype(x + r) over all of H.
  {
    const int64_t m = m0 + warp;
    float ss = 0.f;
    if (m < p.M) {
      for (int64_t k = lane; k < p.H; k += 32) {
        uint16_t hb = p.x[m * p.ldx + k];
        if (p.r) hb = add_rne1<T>(hb, p.r[m * p.ldr + k]);
        const float hf = Elem<T>::to_f(hb);
        ss = __fadd_rn(ss, __fmul_rn(hf, hf));
        if (blockIdx.x == 0 && p.rout) p.rout[m * p.ldro + k] = hb;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) rstd_s[warp] = row_rstd(ss, p.H, p.eps);
  }
  __syncthreads();

  // Phase 2: re-read, normalise, accumulate.  Thread -> (feature n, two token rows).
  const int tn = tid % BN, tm = (tid / BN) * 2;
  float acc0 = 0.f, acc1 = 0.f;
  for (int64_t k0 = 0; k0 < p.H; k0 += BK) {
    for (int i = tid; i < BM * BK; i += 256) {
      const int mm = i / BK, kk = i % BK;
      const int64_t m = m0 + mm, k = k0 + kk;
      float v = 0.f;
      if (m < p.M && k < p.H) {
        uint16_t hb = p.x[m * p.ldx + k];
        if (p.r) hb = add_rne1<T>(hb, p.r[m * p.ldr + k]);
        const float f = __fmul_rn(__fmul_rn(Elem<T>::to_f(hb), rstd_s[mm]), load_gain(p.g, p.gdt, k));
        v = Elem<T>::to_f(Elem<T>::from_f(f));
      }
      nrm[mm][kk] = v;
    }
    for (int i = tid; i < BN * BK; i += 256) {
      const int nn = i / BK, kk = i % BK;
      const int64_t n = n0 + nn, k = k0 + kk;
      wt[nn][kk] = (n < p.N && k < p.H) ? Elem<T>::to_f(p.w[n * p.ldw + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < BK; ++kk) {
      const float wv = wt[tn][kk];
      acc0 = fmaf(nrm[tm][kk], wv, acc0);
      acc1 = fmaf(nrm[tm + 1][kk], wv, acc1);
    }
    __syncthreads();
  }
  const int64_t n = n0 + tn;
  if (n < p.N) {
    if (m0 + tm < p.M) p.out[(m0 + tm) * p.ldo + n] = Elem<T>::from_f(acc0);
    if (m0 + tm + 1 < p.M) p.out[(m0 + tm + 1) * p.ldo + n] = Elem<T>::from_f(acc1);
  }
}

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
cudaError_t launch_prepass(const PrepassParams& p, bool bf16, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)p.M);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const int64_t cpt = (p.H / 8 + 255) / 256;
  if (cpt <= 1)
    return bf16 ? cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__nv_bfloat16, 1>, p)
                : cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__half, 1>, p);
  if (cpt <= 2)
    return bf16 ? cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__nv_bfloat16, 2>, p)
                : cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__half, 2>, p);
  if (cpt <= 4)
    return bf16 ? cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__nv_bfloat16, 4>, p)
                : cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__half, 4>, p);
  return bf16 ? cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__nv_bfloat16, 8>, p)
              : cudaLaunchKernelEx(&cfg, norm_prepass_kernel<__half, 8>, p);
}

cudaError_t launch_simt(const SimtParams& p, bool bf16, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)((p.N + 63) / 64), (unsigned)((p.M + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return bf16 ? cudaLaunchKernelEx(&cfg, simt_kernel<__nv_bfloat16>, p)
              : cudaLaunchKernelEx(&cfg, simt_kernel<__half>, p);
}

}  // namespace fqkv
