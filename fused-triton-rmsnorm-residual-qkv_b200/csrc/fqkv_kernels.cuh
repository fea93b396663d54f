// fqkv_kernels.cuh -- parameter blocks, element-wise helpers and host launcher
// declarations shared by the kernels of the fused RMSNorm+QKV library.
#pragma once

#include <cuda_runtime.h>

#include "fqkv_device.cuh"

namespace fqkv {

// ------------------------------------------------------------------ parameters
// Packed projection output -> head-major Q, K, V with the rotary embedding on Q and K
// (fqkv_rope.cu).  Rows m = b * S + s of qkv hold [Q heads | K heads | V heads].
struct RopeParams {
  const uint16_t* qkv;        // [M, (n_q + 2 n_kv) * head_dim], row stride ldq
  const uint16_t* cos;        // [B or 1, S, head_dim]
  const uint16_t* sin;        // same layout as cos
  uint16_t* q;                // [B, n_q, S, head_dim]
  uint16_t* k;                // [B, n_kv, S, head_dim]
  uint16_t* v;                // [B, n_kv, S, head_dim]
  int64_t M, S, ldq;
  int64_t cs_batch_stride;    // S * head_dim, or 0 when cos / sin are shared by the batch
  int n_q, n_kv, head_dim;
};

struct PrepassParams {
  const uint16_t* x;
  const uint16_t* r;  // nullable
  const void* g;
  int gdt;
  uint16_t* rout;     // nullable
  uint16_t* normed;   // [M, H], row stride H
  int64_t M, H;
  int64_t ldx, ldr, ldro;
  float eps;
  int* counters;      // nullable: zeroed by CTA 0 (the stream-K GEMM's arrival counters)
  int n_counters;
};

struct SimtParams {
  const uint16_t* x;
  const uint16_t* r;  // nullable
  const void* g;
  int gdt;
  const uint16_t* w;
  uint16_t* out;
  uint16_t* rout;     // nullable
  int64_t M, H, N;
  int64_t ldx, ldr, ldw, ldo, ldro;
  float eps;
};

struct DecodeParams {
  const uint16_t* x;
  const uint16_t* r;  // nullable
  const void* g;
  int gdt;
  uint16_t* out;
  uint16_t* rout;     // nullable
  int M, H, N;
  int64_t ldx, ldr, ldo, ldro;
  float eps;
  int kb_total;       // ceil(H / 64)
  int nkb_max;        // max k-blocks of one CTA's K slice
  int flags;
  int pre_stages;     // weight stages issued before the activation loads are out
  int recv_in_normed; // the epilogue's receive slots use the (then idle) normalised-activation
                      // buffer instead of the ring
  const float* wscale;  // e4m3 weights: fp32 scale per weight row (output feature); else null
  // Grid variant (no cluster): per-CTA partial slots [groups][S][M][NT * 128] fp32 and one
  // arrival counter per tile group (zero on entry, left zero on exit).
  float* gpart;
  int* gcnt;
  // Rotary split (cluster kernel, 16-bit weights, own receive slots): with q set, the output
  // is written head-major as q [B, n_q, S, d], k and v [B, n_kv, S, d] (token m = b * S + s),
  // with the rotary embedding on q and k (cos / sin [B or 1, S, d]), instead of `out`.
  uint16_t* q;
  uint16_t* k;
  uint16_t* v;
  const uint16_t* cos;
  const uint16_t* sin;
  int64_t S, cs_batch_stride;
  int n_q, n_kv, head_dim;
};

struct StreamKParams {
  uint16_t* out;
  float* partials;    // [grid][2][MPAD][128] fp32 partial tiles
  int* counters;      // [tiles] arrival counters, zero on entry
  int M, N, H;
  int64_t ldo;
  int kb_total;
  int tiles;
  int flags;
  int b_slots;        // > 0: normalised rows resident in shared memory (slots of MPAD x 64)
  int w_evict_first;  // weight loads carry an L2 evict-first hint
};

struct GemmParams {
  uint16_t* out;
  int M, N, H;
  int64_t ldo;
  int kb_total;
  int tiles_m, tiles_n;
  int flags;
  // CTA-pair kernel: 1 when tmO maps `out` (16-byte aligned address and row pitch) and
  // tiles leave through TMA tensor stores; 0 for per-thread stores.
  int out_tma;
};

// ------------------------------------------------------------------ element helpers
// h = dtype(fp32(x) + fp32(r)), round to nearest even: PyTorch's add of two
// half-precision tensors (baseline.py:48).
template <typename T>
__device__ __forceinline__ uint16_t add_rne1(uint16_t a, uint16_t b) {
  return Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(a), Elem<T>::to_f(b)));
}

template <typename T>
__device__ __forceinline__ uint32_t add_rne2(uint32_t a, uint32_t b) {
  return Elem<T>::from_f2(__fadd_rn(Elem<T>::to_f((uint16_t)(a & 0xFFFFu)), Elem<T>::to_f((uint16_t)(b & 0xFFFFu))),
                          __fadd_rn(Elem<T>::to_f((uint16_t)(a >> 16)), Elem<T>::to_f((uint16_t)(b >> 16))));
}

template <typename T>
__device__ __forceinline__ uint4 add_rne8(uint4 a, uint4 b) {
  return make_uint4(add_rne2<T>(a.x, b.x), add_rne2<T>(a.y, b.y), add_rne2<T>(a.z, b.z), add_rne2<T>(a.w, b.w));
}

// ------------------------------------------------------------------ packed fp32x2
// Two fp32 values in one 64-bit register (element k in the low half, k + 1 in the high
// half) for sm_100's fp32x2 instructions: one instruction, two IEEE round-to-nearest
// results, so the values are those of the scalar __fmul_rn / __fmaf_rn.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// The two 16-bit elements of a 32-bit word as an fp32 pair.
template <typename T>
__device__ __forceinline__ uint64_t f2_from_word(uint32_t w);
template <>
__device__ __forceinline__ uint64_t f2_from_word<__nv_bfloat16>(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ uint64_t f2_from_word<__half>(uint32_t w) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  return f2_pack(f.x, f.y);
}

// dtype(x + r) on two elements at once.  A 16-bit add rounded once to nearest even gives
// the same bits as rounding the fp32 sum to the 16-bit type (what add_rne1 computes): the
// fp32 sum of two bf16 values is exact unless their exponents differ by more than 16,
// and of two fp16 values unless they differ by more than 13.  In those cases the smaller
// operand is below 1/8 ulp of the larger, the exact sum is far from a rounding tie, and
// both roundings return the same value.
template <typename T>
__device__ __forceinline__ uint32_t add2_rn(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t add2_rn<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <>
__device__ __forceinline__ uint32_t add2_rn<__half>(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <typename T>
__device__ __forceinline__ uint4 add8_rn(uint4 a, uint4 b) {
  return make_uint4(add2_rn<T>(a.x, b.x), add2_rn<T>(a.y, b.y), add2_rn<T>(a.z, b.z), add2_rn<T>(a.w, b.w));
}

// acc (an fp32 pair) + squares of the 8 elements: even elements in the low half, odd
// in the high half, fused multiply-adds in element order.
template <typename T>
__device__ __forceinline__ uint64_t sumsq8_f2(uint4 v, uint64_t acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t e = f2_from_word<T>(w[i]);
    acc = f2_fma(e, e, acc);
  }
  return acc;
}

// dtype((fp32(h) * rstd) * g) on 8 elements; rs2 = {rstd, rstd}, g2[i] = gain pair of
// elements 2i, 2i + 1.  Same roundings, in the same order, as normalize1.
template <typename T>
__device__ __forceinline__ uint4 normalize8_f2(uint4 h, uint64_t rs2, const uint64_t (&g2)[4]) {
  const uint32_t w[4] = {h.x, h.y, h.z, h.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lo, hi;
    f2_unpack(f2_mul(f2_mul(f2_from_word<T>(w[i]), rs2), g2[i]), lo, hi);
    o[i] = Elem<T>::from_f2(lo, hi);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Largest magnitude of 8 elements as its 16-bit pattern: fp16 and bf16 magnitudes order like
// their bit patterns with the sign cleared, so a packed unsigned max of (bits & 0x7FFF)
// finds it (a NaN's pattern is above every finite value's).
__device__ __forceinline__ uint32_t absmax8_bits(uint4 v, uint32_t m2) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) asm("max.u16x2 %0, %0, %1;" : "+r"(m2) : "r"(w[i] & 0x7FFF7FFFu));
  return m2;
}

// Two elements of a 16-bit word times `up` (a power of two), as an f16x2 word: exact for
// every product of 2^-17 or more in magnitude (8 or 11 significant bits), and the products
// are below 256.  What is smaller lies below half of e4m3's smallest subnormal (2^-10) and
// adds no e4m3 term either way.
template <typename T>
__device__ __forceinline__ uint32_t scaled_f16x2(uint32_t w, float up) {
  const float lo = Elem<T>::to_f((uint16_t)(w & 0xFFFFu)) * up;
  const float hi = Elem<T>::to_f((uint16_t)(w >> 16)) * up;
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// 8 elements times `up` (a power of two) as K e4m3 terms, one 8-byte group each (element e
// in byte e): term t is the value left by terms 0 .. t-1, rounded to e4m3 (the hardware
// conversion, round to nearest even, saturating).  The values and what is left stay in
// f16x2 words: each difference of a value and its e4m3 rounding is exact there.  With
// |value * up| < 256, two terms hold a bf16 value and three an fp16 value exactly, but for
// what falls below e4m3's smallest subnormal, 2^-9 (values 2^16 times below the row's
// largest and smaller).
template <typename T, int K>
__device__ __forceinline__ void split_e4m3(uint4 v, float up, uint2 (&out)[K]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = scaled_f16x2<T>(w[i], up);
#pragma unroll
  for (int t = 0; t < K; ++t) {
    uint32_t b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint16_t q;
      asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(q) : "r"(r[i]));
      b[i] = q;
      if (t + 1 < K) {
        uint32_t back;
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(back) : "h"(q));
        asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(r[i]) : "r"(back));
      }
    }
    out[t] = make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
  }
}

// ss + sum of squares of the 8 elements, in element order.
template <typename T>
__device__ __forceinline__ float sumsq8_acc(uint4 v, float ss) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = Elem<T>::to_f((uint16_t)(w[i] & 0xFFFFu));
    const float hi = Elem<T>::to_f((uint16_t)(w[i] >> 16));
    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
  }
  return ss;
}

// dtype((fp32(h) * rstd) * fp32(g[k])), the order of baseline.py:61-62 / kernel.py:204.
template <typename T>
__device__ __forceinline__ uint16_t normalize1(uint16_t h, float rstd, float g) {
  return Elem<T>::from_f(__fmul_rn(__fmul_rn(Elem<T>::to_f(h), rstd), g));
}

template <typename T>
__device__ __forceinline__ uint4 normalize8(uint4 h, float rstd, const void* g, int gdt, int64_t k) {
  const uint32_t w[4] = {h.x, h.y, h.z, h.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint16_t lo = normalize1<T>((uint16_t)(w[i] & 0xFFFFu), rstd, load_gain(g, gdt, k + 2 * i));
    const uint16_t hi = normalize1<T>((uint16_t)(w[i] >> 16), rstd, load_gain(g, gdt, k + 2 * i + 1));
    o[i] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Gain elements k .. k+7 as fp32, one or two vector loads (k a multiple of 8; the gain
// row is 16-byte aligned).
__device__ __forceinline__ void load_gain8(const void* g, int gdt, int64_t k, float4 (&out)[2]) {
  if (gdt == FQKV_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(g) + k);
    out[0] = __ldg(p);
    out[1] = __ldg(p + 1);
    return;
  }
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(g) + k));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint16_t lo = (uint16_t)(w[i] & 0xFFFFu), hi = (uint16_t)(w[i] >> 16);
    f[2 * i] = gdt == FQKV_BF16 ? Elem<__nv_bfloat16>::to_f(lo) : Elem<__half>::to_f(lo);
    f[2 * i + 1] = gdt == FQKV_BF16 ? Elem<__nv_bfloat16>::to_f(hi) : Elem<__half>::to_f(hi);
  }
  out[0] = make_float4(f[0], f[1], f[2], f[3]);
  out[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// The 16 bytes (bf16/fp16) or 32 bytes (fp32) of gain elements k .. k+7, raw; converted
// later by gain_raw_to_f32 so that issuing the loads never waits for them.
__device__ __forceinline__ void load_gain8_raw(const void* g, int gdt, int64_t k, uint4 (&raw)[2]) {
  if (gdt == FQKV_F32) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(g) + k);
    raw[0] = __ldg(p);
    raw[1] = __ldg(p + 1);
  } else {
    raw[0] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(g) + k));
    raw[1] = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void gain_raw_to_f32(int gdt, const uint4 (&raw)[2], float4 (&out)[2]) {
  if (gdt == FQKV_F32) {
    out[0] = make_float4(__uint_as_float(raw[0].x), __uint_as_float(raw[0].y), __uint_as_float(raw[0].z),
                         __uint_as_float(raw[0].w));
    out[1] = make_float4(__uint_as_float(raw[1].x), __uint_as_float(raw[1].y), __uint_as_float(raw[1].z),
                         __uint_as_float(raw[1].w));
    return;
  }
  const uint32_t w[4] = {raw[0].x, raw[0].y, raw[0].z, raw[0].w};
  float f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint16_t lo = (uint16_t)(w[i] & 0xFFFFu), hi = (uint16_t)(w[i] >> 16);
    f[2 * i] = gdt == FQKV_BF16 ? Elem<__nv_bfloat16>::to_f(lo) : Elem<__half>::to_f(lo);
    f[2 * i + 1] = gdt == FQKV_BF16 ? Elem<__nv_bfloat16>::to_f(hi) : Elem<__half>::to_f(hi);
  }
  out[0] = make_float4(f[0], f[1], f[2], f[3]);
  out[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// normalize8 with the gain already in registers.
template <typename T>
__device__ __forceinline__ uint4 normalize8g(uint4 h, float rstd, const float4 (&g)[2]) {
  const float gf[8] = {g[0].x, g[0].y, g[0].z, g[0].w, g[1].x, g[1].y, g[1].z, g[1].w};
  const uint32_t w[4] = {h.x, h.y, h.z, h.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __fmul_rn(__fmul_rn(Elem<T>::to_f((uint16_t)(w[i] & 0xFFFFu)), rstd), gf[2 * i]);
    const float hi = __fmul_rn(__fmul_rn(Elem<T>::to_f((uint16_t)(w[i] >> 16)), rstd), gf[2 * i + 1]);
    o[i] = Elem<T>::from_f2(lo, hi);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ------------------------------------------------------------------ launchers
// Raise a kernel's dynamic shared-memory limit to `bytes` (cached per kernel and device).
cudaError_t ensure_smem_attr(const void* func, size_t bytes);

cudaError_t launch_prepass(const PrepassParams& p, bool bf16, bool pdl, cudaStream_t stream);
cudaError_t launch_simt(const SimtParams& p, bool bf16, bool pdl, cudaStream_t stream);

// Fused decode schedule chosen on the host.
// Threads of the fused decode kernel: a TMA producer warp, an MMA warp, 8 norm/epilogue warps.
constexpr int kDecodeThreads = 64 + 8 * 32;

struct DecodeConfig {
  int mpad;     // token columns of the MMA (16, 32 or 64)
  int nt;       // 128-row W tiles per CTA (1 to 5)
  int stages;   // ring depth
  int cluster;  // CTAs splitting K (cluster size)
  size_t smem;  // dynamic shared memory bytes
  int recv_in_normed;  // see DecodeParams
  int f8;       // e4m3 weights: the e4m3 terms each activation is split into (2 for bf16,
                // 3 for fp16); 0 for 16-bit weights
  int grid;     // 1: `cluster` independent CTAs split K (no cluster); they sum their partial
                // tiles through the workspace
};

// e4m3 terms that hold a normalised 16-bit activation exactly (8 or 11 significant bits).
__host__ __device__ constexpr int decode_f8_terms(bool bf16) { return bf16 ? 2 : 3; }
// The K slice of rank r of the C CTAs splitting KB 64-deep k-blocks: [begin(r), begin(r + 1)).
// e4m3 weights split in units of two k-blocks (one ring stage of 128 one-byte columns), so
// that no CTA streams a half-empty stage.
__host__ __device__ constexpr int decode_slice_begin(int r, int C, int KB, bool f8) {
  return f8 ? (2 * ((r * ((KB + 1) / 2)) / C) < KB ? 2 * ((r * ((KB + 1) / 2)) / C) : KB) : (r * KB) / C;
}
__host__ __device__ constexpr int decode_slice_max(int C, int KB, bool f8) {
  return f8 ? 2 * (((KB + 1) / 2 + C - 1) / C) : (KB + C - 1) / C;
}
// f8: 0 for 16-bit weights, else decode_f8_terms of the activation dtype.
int decode_pick_config(int M, int H, int N, int sm_count, DecodeConfig* cfg, int f8 = 0);
// DecodeConfig::recv_in_normed value of the receive slots in a region of their own (the
// epilogue needs no cluster agreement before its copies; the rotary split needs these).
constexpr int kDecodeRecvOwn = 2;
constexpr int kDecodeRopeMaxM = 32;  // the rotary-split epilogue: 16-bit weights, own slots
// Grid variant of the fused decode kernel: every CTA reads whole activation rows, so it
// serves few rows only.
constexpr int kGridMaxM = 8;
constexpr int kGridMaxSplit = 8;  // CTAs splitting K per tile group
constexpr int kGridMaxTiles = 1024;  // 128-row tiles (N <= 131072): counters in the workspace
int decode_grid_pick_config(int M, int H, int N, int sm_count, DecodeConfig* cfg);
// Workspace of the grid variant: [kGridMaxTiles arrival counters][partial slots].
int64_t decode_grid_counter_bytes();
int64_t decode_grid_workspace_bytes(int64_t M, int64_t N);
// 128-row weight tiles per TMA box of the decode kernel's weight map: one box per stage
// for NT <= 2, else NT boxes of 128 rows (a box dimension is at most 256 elements).
__host__ __device__ constexpr int decode_box_tiles(int nt) { return nt <= 2 ? nt : 1; }
size_t decode_smem_bytes(const DecodeConfig& c, int kb_total);
cudaError_t launch_decode(const DecodeConfig& c, const CUtensorMap& tmW, const DecodeParams& p, bool bf16, bool pdl,
                          cudaStream_t stream);

constexpr int kStreamKMaxGrid = 320;  // partial-slot capacity of the workspace (>= 2 x SM count)
struct StreamKConfig {
  int mpad;
  int stages;
  int grid;
  int b_slots;
  int w_evict_first;
  size_t smem;
};
int streamk_mpad(int M);
int64_t streamk_partials_bytes(int M);
int64_t streamk_counters_bytes(int N);
int streamk_pick_config(int M, int H, int N, int sm_count, StreamKConfig* cfg);
cudaError_t launch_streamk(const StreamKConfig& c, const CUtensorMap& tmW, const CUtensorMap& tmB,
                           const StreamKParams& p, bool bf16, bool pdl, cudaStream_t stream);

struct GemmConfig {
  int bn;       // output features per tile (MMA N)
  int stages;
  int grid;
  size_t smem;
  int pair;     // 1: 2-CTA clusters computing 256-row tiles (tcgen05 cta_group::2)
};
int gemm_pick_config(int M, int H, int N, int sm_count, GemmConfig* cfg);
cudaError_t launch_rope_split(const RopeParams& p, bool bf16, cudaStream_t stream);
cudaError_t launch_gemm(const GemmConfig& c, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                        const GemmParams& p, bool bf16, bool pdl, cudaStream_t stream);

}  // namespace fqkv
