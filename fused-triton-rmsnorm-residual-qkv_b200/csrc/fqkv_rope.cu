// fqkv_rope.cu -- the packed projection's output split into head-major Q, K and V, with
// the rotary position embedding applied to Q and K, in one launch.
//
// Replaces what the Llama integration runs after the fused projection (the reference's
// llama3_patch.py:156-168, which calls transformers' apply_rotary_pos_emb): split the
// [M, (n_q + 2 n_kv) d] output by [n_q d, n_kv d, n_kv d], view each part as heads,
// transpose to (B, heads, S, d) and rotate Q and K:
//   x_rot = x * cos + rotate_half(x) * sin,   rotate_half(x) = cat(-x[d/2:], x[:d/2]).
// The arithmetic repeats PyTorch's 16-bit elementwise ops one by one: each product is the
// fp32 product rounded to the dtype, and the sum is the fp32 sum of the two rounded
// products, rounded to the dtype -- so the result is bit-identical to that sequence.
//
// One thread per (token, head, 8-element group of the first half): it reads 16 bytes of
// each half of the head, and of cos and sin at both halves, and writes 16 bytes to each
// half of the head's row in the head-major output.  HBM-bound (every byte moves once).
#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

template <typename T>
__device__ __forceinline__ float rd(uint16_t v) {
  return Elem<T>::to_f(v);
}

// dtype(dtype(a * c) + dtype(b * s)): PyTorch's a * c + b * s on 16-bit tensors.
template <typename T>
__device__ __forceinline__ uint16_t mul_add_16(uint16_t a, uint16_t c, uint16_t b, uint16_t s) {
  const uint16_t p = Elem<T>::from_f(__fmul_rn(rd<T>(a), rd<T>(c)));
  const uint16_t q = Elem<T>::from_f(__fmul_rn(rd<T>(b), rd<T>(s)));
  return Elem<T>::from_f(__fadd_rn(rd<T>(p), rd<T>(q)));
}

template <typename T>
__global__ void __launch_bounds__(256) rope_split_kernel(const RopeParams p) {
  const int d = p.head_dim, half = d / 2, groups = half / 8;
  const int heads = p.n_q + 2 * p.n_kv;
  const int64_t total = p.M * heads * groups;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(t % groups);
    const int h = (int)((t / groups) % heads);
    const int64_t m = t / ((int64_t)groups * heads);
    const int64_t b = m / p.S, s = m % p.S;
    const uint16_t* src = p.qkv + m * p.ldq + (int64_t)h * d + g * 8;
    uint16_t x1[8], x2[8];
    *reinterpret_cast<uint4*>(x1) = *reinterpret_cast<const uint4*>(src);
    *reinterpret_cast<uint4*>(x2) = *reinterpret_cast<const uint4*>(src + half);
    uint16_t* dst;
    if (h < p.n_q) {
      dst = p.q + ((b * p.n_q + h) * p.S + s) * d;
    } else if (h < p.n_q + p.n_kv) {
      dst = p.k + ((b * p.n_kv + (h - p.n_q)) * p.S + s) * d;
    } else {
      dst = p.v + ((b * p.n_kv + (h - p.n_q - p.n_kv)) * p.S + s) * d;
    }
    uint16_t o1[8], o2[8];
    if (h < p.n_q + p.n_kv) {
      const int64_t cs = b * p.cs_batch_stride + s * d + g * 8;
      uint16_t c1[8], c2[8], s1[8], s2[8];
      *reinterpret_cast<uint4*>(c1) = *reinterpret_cast<const uint4*>(p.cos + cs);
      *reinterpret_cast<uint4*>(c2) = *reinterpret_cast<const uint4*>(p.cos + cs + half);
      *reinterpret_cast<uint4*>(s1) = *reinterpret_cast<const uint4*>(p.sin + cs);
      *reinterpret_cast<uint4*>(s2) = *reinterpret_cast<const uint4*>(p.sin + cs + half);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // first half:  x1 * cos + (-x2) * sin;  second half: x2 * cos + x1 * sin
        o1[j] = mul_add_16<T>(x1[j], c1[j], (uint16_t)(x2[j] ^ 0x8000u), s1[j]);
        o2[j] = mul_add_16<T>(x2[j], c2[j], x1[j], s2[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o1[j] = x1[j];
        o2[j] = x2[j];
      }
    }
    *reinterpret_cast<uint4*>(dst + g * 8) = *reinterpret_cast<const uint4*>(o1);
    *reinterpret_cast<uint4*>(dst + half + g * 8) = *reinterpret_cast<const uint4*>(o2);
  }
}

}  // namespace

cudaError_t launch_rope_split(const RopeParams& p, bool bf16, cudaStream_t stream) {
  const int64_t total = p.M * (p.n_q + 2 * p.n_kv) * (p.head_dim / 16);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 blocks per SM
  if (blocks < 1) blocks = 1;
  if (bf16)
    rope_split_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(p);
  else
    rope_split_kernel<__half><<<(unsigned)blocks, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace fqkv
