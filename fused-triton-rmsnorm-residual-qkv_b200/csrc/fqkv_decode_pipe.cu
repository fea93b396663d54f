// fqkv_decode_pipe.cu -- the fused small-M (decode) kernel, pipelined across launches:
// residual add, RMSNorm and the projection in one launch (swap-AB tcgen05 GEMM, K split
// across a thread-block cluster), laid out so that consecutive launches in a stream keep
// HBM busy through each other's start-up and wind-down.
//
// Decode reads the whole weight once and little else, so a launch is HBM-bound, and the
// time it loses is at its two ends: before the first MMA (activation loads, the cluster's
// exchange of row sums of squares, normalisation) and after the last one (the split-K
// reduction and the stores).  Three things keep those ends off the weight stream:
//   * Weight k-blocks do not depend on the preceding grid.  With static weights the
//     producer fills the whole ring while that grid is still running (the activation loads
//     cannot start before it completes anyway), and only from the moment it has completed
//     does it hold back to `pre` stages until the activations are in.
//   * Each CTA accumulates its NT row tiles one after the other, so the reduction of tile
//     t runs while tile t + 1 streams.
//   * Every tile has one owner CTA in the cluster (rank t % C).  The other CTAs send their
//     fp32 partial of it (tokens m < M only) by one bulk copy into a receive slot of the
//     owner's shared memory, and the owner sums the C partials in rank order
//     (deterministic) and stores the tile.  A CTA that owns no tile is done once its
//     copies have been read; the cluster's last barrier completes when every partial has
//     landed, so such CTAs leave before the owners' sums and stores, and the next launch's
//     CTAs can take their SMs.
//
// Grid = (C, groups), cluster = (C, 1, 1).  CTA `rank` of cluster blockIdx.y owns the K
// slice [kb0, kb1) (64-element k-blocks) of the group's NT 128-row weight tiles.
// Warp roles (320 threads):
//   warp 0     TMA producer: a ring of 128 x 64 weight boxes (16 KB, 128-byte swizzle),
//              tile-major (all k-blocks of tile 0, then tile 1, ...).  No multicast.
//   warp 1     TMEM allocator; lane 0 waits for the preceding grid (and tells the producer
//              when it has completed), then issues the MMAs (tcgen05.mma kind::f16, fp32
//              accumulators in TMEM, one per tile) and commits each tile to its barrier.
//   warps 2-9  norm: h = dtype(x + r) (bit-exact, baseline.py:48), the updated residual
//              (tile group 0), row sums of squares exchanged across the cluster through
//              DSMEM (st.async), normed = dtype((h * rstd) * g) (baseline.py:59-62) into
//              shared memory as the MMA's B operand; then the per-tile epilogue above.
//              With a rotary table the owner writes head-major Q, K, V with the rotary
//              embedding on Q and K (the llama3_patch.py:156-168 sequence, bit-identical to
//              the separate split kernel, fqkv_rope.cu) instead of the packed output.
// Every wait is bounded (fqkv_device.cuh).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

constexpr int kNormWarps = 8;
constexpr int kNormThreads = kNormWarps * 32;
constexpr int kThreads = 64 + kNormThreads;
static_assert(kThreads == kDecodeThreads, "fqkv_kernels.cuh states the decode kernels' block size");
static_assert(5 * 32 <= 256, "NT * MPAD accumulator columns stay within 256 (two CTAs per SM share 512)");
constexpr int kMaxCluster = 8;
constexpr int kTileRows = 128;
constexpr int kKBlock = 64;
constexpr int kBoxBytes = kTileRows * 128;  // one 128 x 64 16-bit weight box
constexpr int kLoadBatch = 4;               // 16-byte chunks per lane and row loaded before any is used
constexpr int kGainChunks = 2;              // gain chunks per thread: K slices up to 2 * 256 * 8 elements
constexpr int kMaxNT = 5;

struct PLayout {
  uint32_t ring, normed, gain, red, rowp, rstd, stage, recv, tout, bars, misc, total;
};

// Shared memory of one CTA.  `own_max` tiles owned per CTA, `cl` CTAs in the cluster.
__host__ __device__ inline PLayout make_pipe_layout(int stages, int nt, int mpad, int nkb_max, int cl) {
  PLayout L;
  const int own_max = (nt + cl - 1) / cl;
  L.ring = 0;
  L.normed = L.ring + stages * kBoxBytes;                 // 1024-aligned
  L.gain = L.normed + (uint32_t)nkb_max * mpad * 128;     // [nkb_max * 64] fp32
  L.red = L.gain + (uint32_t)nkb_max * kKBlock * 4;       // [kMaxCluster][mpad] fp32
  L.rowp = L.red + kMaxCluster * mpad * 4;
  L.rstd = L.rowp + mpad * 4;
  L.stage = (L.rstd + mpad * 4 + 127) & ~127u;            // [nt][mpad][128] fp32 partials to send
  L.recv = L.stage + (uint32_t)nt * mpad * kTileRows * 4;  // [own_max][cl - 1][mpad][128] fp32
  L.tout = L.recv + (uint32_t)own_max * (cl - 1) * mpad * kTileRows * 4;  // [mpad][128] dtype
  L.bars = (L.tout + mpad * kTileRows * 2 + 7) & ~7u;     // full[S] empty[S] acc[nt] normed sum acts recv[own]
  L.misc = L.bars + (2 * stages + nt + 3 + own_max) * 8;  // tmem base, producer flag
  L.total = L.misc + 16;
  return L;
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32u : cols <= 64 ? 64u : cols <= 128 ? 128u : cols <= 256 ? 256u : 512u;
}

// 32 lanes x 32 bits, 8 consecutive columns: thread i receives TMEM[lane_base + i][col .. col+7].
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ uint32_t ld_volatile_shared(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_shared(uint32_t* p, uint32_t v) {
  asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ float rd16(uint16_t v) {
  return Elem<T>::to_f(v);
}

// dtype(dtype(a * c) + dtype(b * s)): PyTorch's a * c + b * s on 16-bit tensors (the
// rounding sequence of fqkv_rope.cu).
template <typename T>
__device__ __forceinline__ uint16_t rope_mul_add(uint16_t a, uint16_t c, uint16_t b, uint16_t s) {
  const uint16_t p = Elem<T>::from_f(__fmul_rn(rd16<T>(a), rd16<T>(c)));
  const uint16_t q = Elem<T>::from_f(__fmul_rn(rd16<T>(b), rd16<T>(s)));
  return Elem<T>::from_f(__fadd_rn(rd16<T>(p), rd16<T>(q)));
}

template <typename T, int MPAD, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    pipe_decode_kernel(const __grid_constant__ CUtensorMap tmW, const PipeParams p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  FQKV_TRACE_DECL
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t C = gridDim.x;
  const uint32_t rank = cluster_ctarank();
  const PLayout L = make_pipe_layout(stages, NT, MPAD, p.nkb_max, (int)C);
  const int own_max = (NT + (int)C - 1) / (int)C;
  uint8_t* ring = smem + L.ring;
  uint8_t* normed = smem + L.normed;
  float* gain_s = reinterpret_cast<float*>(smem + L.gain);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* rowp = reinterpret_cast<float*>(smem + L.rowp);
  float* rstd_s = reinterpret_cast<float*>(smem + L.rstd);
  float* stage_s = reinterpret_cast<float*>(smem + L.stage);
  float* recv_s = reinterpret_cast<float*>(smem + L.recv);
  uint16_t* tout = reinterpret_cast<uint16_t*>(smem + L.tout);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  uint64_t* acc_bar = empty + stages;    // [NT]: tile nt's MMAs have completed
  uint64_t* normed_bar = acc_bar + NT;   // the normalised activations are in shared memory
  uint64_t* sum_bar = normed_bar + 1;    // the cluster's row sums of squares have landed
  uint64_t* acts_bar = normed_bar + 2;   // the activation loads have returned
  uint64_t* recv_bar = normed_bar + 3;   // [own_max]: the peers' partials of an owned tile have landed
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L.misc);  // [0] TMEM base, [1] preceding grid done

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.kb_total;
  const int kb0 = (int)((rank * (uint32_t)KB) / C), kb1 = (int)(((rank + 1) * (uint32_t)KB) / C);
  const int nkb = kb1 - kb0;
  const int n_base = blockIdx.y * NT * kTileRows;
  constexpr uint32_t kTmemCols = tmem_cols_for(NT * MPAD);
  const uint32_t part_bytes = (uint32_t)p.M * kTileRows * 4;  // one CTA's partial of one tile

  // ---------------------------------------------------------------- setup
  FQKV_TRACE_BEGIN();
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < NT; ++t) mbar_init(&acc_bar[t], 1);
    mbar_init(normed_bar, 1);
    mbar_init(sum_bar, 1);   // local arrive + C * MPAD * 4 bytes of st.async from the cluster
    mbar_init(acts_bar, 1);
    for (int o = 0; o < own_max; ++o) mbar_init(&recv_bar[o], 1);  // local arrive + the peers' copies
    misc[1] = 0;
    fence_mbarrier_init_cluster();
    FQKV_TRACE_POINT(17);
    // Announce the incoming bytes before any peer can send them (peers send after the
    // cluster barrier below).
    mbar_arrive_expect_tx_cluster(sum_bar, C * MPAD * 4);
    for (int t = (int)rank; t < NT; t += (int)C) mbar_arrive_expect_tx_cluster(&recv_bar[t / C], (C - 1) * part_bytes);
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmW);
  if (warp == 1) {
    tmem_alloc(misc, kTmemCols);
    tmem_relinquish();
    if (lane == 0) FQKV_TRACE_POINT(18);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(misc);
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (threadIdx.x == 0) FQKV_TRACE_POINT(3);
  const bool static_w = (p.flags & FQKV_FLAG_STATIC_WEIGHTS) != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      if (!static_w) pdl_wait();
      const int total = NT * nkb;
      const int pre = min(total, min(stages, p.pre_stages));
      const uint64_t pol_w = policy_evict_first();
      bool ok = true, acts_in = false;
      int s = 0, round = 0, issued = 0;
      for (int j = 0; j < total; ++j) {
        // Beyond `pre` stages, the weight flood would queue ahead of the activation loads;
        // those start once the preceding grid has completed, so until then the ring fills.
        if (!acts_in && j >= pre && (round > 0 || ld_volatile_shared(&misc[1]) != 0)) {
          ok = mbar_wait(acts_bar, 0);
          acts_in = true;
          FQKV_TRACE_POINT(5);
        }
        if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1))) break;
        const int nt = j / nkb, i = j - nt * nkb;
        mbar_arrive_expect_tx(&full[s], kBoxBytes);
        tma_load_2d_hint(ring + s * kBoxBytes, &tmW, &full[s], (kb0 + i) * kKBlock, n_base + nt * kTileRows, pol_w);
        if (j == 0) FQKV_TRACE_POINT(4);
        ++issued;
        if (++s == stages) {
          s = 0;
          ++round;
        }
      }
      FQKV_TRACE_POINT(6);
      // None of this CTA's loads may still be in flight when it leaves: only the last
      // `stages` can be (bounded waits).
      for (int j = max(0, issued - stages); j < issued; ++j) mbar_wait(&full[j % stages], (j / stages) & 1);
      (void)ok;
    }
    __syncwarp();
    cluster_arrive_release_thread();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      pdl_wait();
      st_volatile_shared(&misc[1], 1u);  // the preceding grid has completed
      const uint32_t idesc = make_idesc_f16(kTileRows, MPAD, std::is_same<T, __nv_bfloat16>::value);
      bool ok = mbar_wait(normed_bar, 0);
      int s = 0, round = 0;
      for (int nt = 0; nt < NT; ++nt) {
        for (int i = 0; i < nkb && ok; ++i) {
          if (!(ok = mbar_wait(&full[s], round & 1))) break;
          if (nt == 0 && i == 0) FQKV_TRACE_POINT(11);
          tc_fence_after();
          const uint32_t a_base = smem_u32(ring + s * kBoxBytes);
          const uint32_t b_base = smem_u32(normed + i * MPAD * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem_base + nt * MPAD, make_sw128_desc(a_base + kk * 32), make_sw128_desc(b_base + kk * 32),
                     idesc, (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
        // Also on failure, so that no epilogue waits for MMAs that never come.
        umma_commit(&acc_bar[nt]);
      }
      FQKV_TRACE_POINT(12);
      mbar_wait(&acc_bar[NT - 1], 0);  // every MMA has retired before TMEM is freed
    }
    __syncwarp();
    tc_fence_before();
    cluster_arrive_release_thread();
  } else {
    // ------------------------------------------------------------ norm (warps 2..9)
    const int et = threadIdx.x - 64;
    const int nw = warp - 2;
    const int nchunk = nkb * 8;  // 16-byte chunks per row of the slice
    const int64_t k_lo = (int64_t)kb0 * kKBlock;
    const bool write_res = p.rout != nullptr && blockIdx.y == 0;
    bool ok = true;
    uint4 graw[kGainChunks][2];
    auto issue_gain = [&]() {
#pragma unroll
      for (int i = 0; i < kGainChunks; ++i) {
        const int j = et + kNormThreads * i;
        const int64_t k = k_lo + (int64_t)j * 8;
        graw[i][0] = graw[i][1] = make_uint4(0, 0, 0, 0);
        if (j < nchunk && k < p.H) load_gain8_raw(p.g, p.gdt, k, graw[i]);
      }
    };
    if (static_w) issue_gain();
    // Warm L2 with this CTA's slice of x and the residual while the preceding grid may still
    // run (a prefetch loads nothing into registers; a later write of that grid lands in L2).
    if (p.M > 1) {
      const int nline = (nchunk + 7) >> 3;
      for (int t = et; t < p.M * nline; t += kNormThreads) {
        const int m = t / nline;
        const int64_t k = k_lo + (int64_t)(t - m * nline) * 64;
        if (k < p.H) {
          prefetch_l2(p.x + (int64_t)m * p.ldx + k);
          if (p.r) prefetch_l2(p.r + (int64_t)m * p.ldr + k);
        }
      }
    }
    pdl_wait();
    if (et == 0) FQKV_TRACE_POINT(7);
    if (!static_w) issue_gain();
    // Pass 1: warp nw takes rows nw and nw + 8 (then + 16, + 24 for MPAD 32); each lane issues
    // up to kLoadBatch chunk loads of x (and r) per row before consuming any.
    const bool h_in_regs = MPAD == 2 * kNormWarps && nchunk <= 32 * kLoadBatch;
    uint4 hkeep[2][kLoadBatch];
    for (int m0 = nw; m0 < MPAD; m0 += 2 * kNormWarps) {
      uint64_t ss2[2] = {0ull, 0ull};
      for (int j0 = 0; j0 < nchunk; j0 += 32 * kLoadBatch) {
        uint4 xv[2][kLoadBatch], rv[2][kLoadBatch];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int m = m0 + kNormWarps * q2;
          const bool live = m < p.M;
          const uint16_t* xr = p.x + (int64_t)m * p.ldx;
          const uint16_t* rr = p.r ? p.r + (int64_t)m * p.ldr : nullptr;
#pragma unroll
          for (int b = 0; b < kLoadBatch; ++b) {
            const int j = j0 + lane + 32 * b;
            const int64_t k = k_lo + (int64_t)j * 8;
            xv[q2][b] = make_uint4(0, 0, 0, 0);
            rv[q2][b] = make_uint4(0, 0, 0, 0);
            if (live && j < nchunk && k < p.H) {
              xv[q2][b] = __ldg(reinterpret_cast<const uint4*>(xr + k));
              if (rr) rv[q2][b] = __ldg(reinterpret_cast<const uint4*>(rr + k));
            }
          }
        }
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int m = m0 + kNormWarps * q2;
          const bool live = m < p.M;
#pragma unroll
          for (int b = 0; b < kLoadBatch; ++b) {
            const int j = j0 + lane + 32 * b;
            const int64_t k = k_lo + (int64_t)j * 8;
            const uint4 hv = p.r ? add8_rn<T>(xv[q2][b], rv[q2][b]) : xv[q2][b];
            ss2[q2] = sumsq8_f2<T>(hv, ss2[q2]);
            if (write_res && live && j < nchunk && k < p.H)
              *reinterpret_cast<uint4*>(p.rout + (int64_t)m * p.ldro + k) = hv;
            hkeep[q2][b] = hv;
            if (j < nchunk) *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) = hv;
          }
        }
      }
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        float lo, hi;
        f2_unpack(ss2[q2], lo, hi);
        float ss = lo + hi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) rowp[m0 + kNormWarps * q2] = ss;
      }
    }
#pragma unroll
    for (int i = 0; i < kGainChunks; ++i) {
      const int j = et + kNormThreads * i;
      if (j < nchunk) {
        float4 gv[2];
        gain_raw_to_f32(p.gdt, graw[i], gv);
        reinterpret_cast<float4*>(gain_s)[2 * j] = gv[0];
        reinterpret_cast<float4*>(gain_s)[2 * j + 1] = gv[1];
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (et == 0) mbar_arrive(acts_bar);
    if (et == 0) FQKV_TRACE_POINT(8);
    // This CTA's per-row partial sums go into slot `rank` of every CTA of the cluster.
    if (warp == 2) {
      for (uint32_t c = 0; c < C; ++c) {
        const uint32_t bar_c = mapa_shared(smem_u32(sum_bar), c);
        for (int m = lane; m < MPAD; m += 32)
          st_async_f32(mapa_shared(smem_u32(&red[rank * MPAD + m]), c), rowp[m], bar_c);
      }
    }
    ok = mbar_wait<true>(sum_bar, 0);
    for (int m = et; m < MPAD; m += kNormThreads) {
      float tot = 0.f;
      for (uint32_t c = 0; c < C; ++c) tot += red[c * MPAD + m];
      rstd_s[m] = row_rstd(tot, p.H, p.eps);
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (et == 0) FQKV_TRACE_POINT(9);
    // Pass 2: normalise, dtype((h * rstd) * g).
    auto load_g2 = [&](int j, uint64_t (&g2)[4]) {
      const ulonglong2 a = reinterpret_cast<const ulonglong2*>(gain_s)[2 * j];
      const ulonglong2 c = reinterpret_cast<const ulonglong2*>(gain_s)[2 * j + 1];
      g2[0] = a.x;
      g2[1] = a.y;
      g2[2] = c.x;
      g2[3] = c.y;
    };
    if (h_in_regs) {
      uint64_t rs2[2];
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        const float rs = rstd_s[nw + kNormWarps * q2];
        rs2[q2] = f2_pack(rs, rs);
      }
#pragma unroll
      for (int b = 0; b < kLoadBatch; ++b) {
        const int j = lane + 32 * b;
        const bool in = j < nchunk && k_lo + (int64_t)j * 8 < p.H;
        uint64_t g2[4];
        load_g2(j < nchunk ? j : nchunk - 1, g2);
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int m = nw + kNormWarps * q2;
          const uint4 o = normalize8_f2<T>(hkeep[q2][b], rs2[q2], g2);
          if (in && m < p.M) *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) = o;
        }
      }
    } else {
      for (int j0 = 0; j0 < nchunk; j0 += 32 * kLoadBatch) {
        uint64_t g2[kLoadBatch][4];
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          const int j = j0 + lane + 32 * b;
          if (j < nchunk) load_g2(j, g2[b]);
        }
        for (int m = nw; m < p.M; m += kNormWarps) {
          const float rs = rstd_s[m];
          const uint64_t rs2 = f2_pack(rs, rs);
          uint4 hv[kLoadBatch];
#pragma unroll
          for (int b = 0; b < kLoadBatch; ++b) {
            const int j = j0 + lane + 32 * b;
            if (j < nchunk && k_lo + (int64_t)j * 8 < p.H)
              hv[b] = *reinterpret_cast<const uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7));
          }
#pragma unroll
          for (int b = 0; b < kLoadBatch; ++b) {
            const int j = j0 + lane + 32 * b;
            if (j < nchunk && k_lo + (int64_t)j * 8 < p.H)
              *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) =
                  normalize8_f2<T>(hv[b], rs2, g2[b]);
          }
        }
      }
    }
    if (et == 0) FQKV_TRACE_POINT(19);
    fence_proxy_async_smem();
    if (et == 0) FQKV_TRACE_POINT(20);
    __syncwarp();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    // FQKV_FLAG_TEST_WITHHOLD (tests of the failure path): no arrival, so the MMA thread's
    // bounded wait runs out; it then commits no MMA and the kernel winds down as usual.
    if (et == 0 && !(p.flags & FQKV_FLAG_TEST_WITHHOLD)) mbar_arrive(normed_bar);
    if (et == 0) FQKV_TRACE_POINT(10);

    // ------------------------------------------------------------ per-tile epilogue
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;  // the two warps of a quadrant take alternate 8-column chunks
    const int row = q * 32 + lane;
    // Each thread arrives on the cluster's last barrier once this CTA is past its last
    // exchange: for the owner of the last tile, when that tile's partials have landed (before
    // its sum and stores); otherwise after the last send, once thread 0's copies have read
    // their sources.
    bool arrived = false;
    auto arrive_cluster = [&]() {
      if (et == 0) bulk_wait_group_read<0>();  // this CTA's partials have been read by its copies
      tc_fence_before();
      cluster_arrive_release_thread();
      arrived = true;
    };
    for (int nt = 0; nt < NT; ++nt) {
      const bool own = (uint32_t)(nt % (int)C) == rank;
      ok = mbar_wait(&acc_bar[nt], 0) && ok;
      if (et == 0 && nt == NT - 1) FQKV_TRACE_POINT(13);
      tc_fence_after();
      // This thread's values: row `row` of the tile, tokens c0 .. c0 + 7 of each of its chunks.
      constexpr int kChunks = MPAD / 16;  // 8-column chunks per warp
      uint32_t v[kChunks][8];
#pragma unroll
      for (int ch = 0; ch < kChunks; ++ch) {
        const int c0 = (2 * ch + half) * 8;
        tmem_ld8(tmem_base + ((uint32_t)(q * 32) << 16) + nt * MPAD + c0, v[ch]);
      }
      tmem_wait_ld();
      if (!own) {
        // Send: this CTA's partial [m][row] (m < M) to slot `slot` of the owner.
        float* st = stage_s + nt * (MPAD * kTileRows);
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          const int c0 = (2 * ch + half) * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c0 + e < p.M) st[(c0 + e) * kTileRows + row] = __uint_as_float(v[ch][e]);
        }
        tc_fence_before();
        fence_proxy_async_smem();  // the bulk copy reads the partial through the async proxy
        __syncwarp();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (et == 0) {
          const uint32_t owner = (uint32_t)(nt % (int)C);
          const uint32_t slot = rank < owner ? rank : rank - 1;
          const uint32_t dst = smem_u32(recv_s) + ((uint32_t)(nt / (int)C) * (C - 1) + slot) * (MPAD * kTileRows * 4);
          bulk_copy_to_peer(mapa_shared(dst, owner), smem_u32(st), part_bytes,
                            mapa_shared(smem_u32(&recv_bar[nt / (int)C]), owner));
          bulk_commit_group();
        }
        continue;
      }
      tc_fence_before();
      // Own: sum the C partials of each value in rank order.
      if (C > 1) ok = mbar_wait<true>(&recv_bar[nt / (int)C], 0) && ok;
      if (et == 0) FQKV_TRACE_POINT(15);
      if (nt == NT - 1) arrive_cluster();
      const float* rv = recv_s + (size_t)(nt / (int)C) * (C - 1) * (MPAD * kTileRows);
      const int n = n_base + nt * kTileRows + row;
#pragma unroll
      for (int ch = 0; ch < kChunks; ++ch) {
        const int c0 = (2 * ch + half) * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int m = c0 + e;
          if (m >= p.M) continue;
          float acc = 0.f;
          for (uint32_t c = 0; c < C; ++c) {
            const float pv = c == rank ? __uint_as_float(v[ch][e])
                                       : rv[(c < rank ? c : c - 1) * (MPAD * kTileRows) + m * kTileRows + row];
            acc += pv;
          }
          const uint16_t o = Elem<T>::from_f(acc);
          if (p.q == nullptr) {
            if (n < p.N) p.out[(int64_t)m * p.ldo + n] = o;
          } else {
            tout[m * kTileRows + row] = o;
          }
        }
      }
      if (p.q != nullptr) {
        // Head-major Q / K / V with the rotary embedding on Q and K, 8 features per thread.
        __syncwarp();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const int d = p.head_dim, hd = d / 2;
        for (int u = et; u < p.M * (kTileRows / 8); u += kNormThreads) {
          const int m = u / (kTileRows / 8), r8 = (u - m * (kTileRows / 8)) * 8;
          const int nn = n_base + nt * kTileRows + r8;
          if (nn >= p.N) continue;
          const int head = nn / d, j = nn - head * d;  // j % 8 == 0, and the 8 stay in one half
          const int64_t b = m / p.S, s = m - b * p.S;
          uint16_t xv[8], ov[8];
          *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(tout + m * kTileRows + r8);
          uint16_t* dst;
          if (head < p.n_q + p.n_kv) {
            const int pr8 = r8 ^ hd;  // the other half of the same head (same tile: d divides 128)
            uint16_t yv[8], cv[8], sv[8];
            *reinterpret_cast<uint4*>(yv) = *reinterpret_cast<const uint4*>(tout + m * kTileRows + pr8);
            const int64_t cs = b * p.cs_batch_stride + s * d + j;
            *reinterpret_cast<uint4*>(cv) = __ldg(reinterpret_cast<const uint4*>(p.cos + cs));
            *reinterpret_cast<uint4*>(sv) = __ldg(reinterpret_cast<const uint4*>(p.sin + cs));
            const bool first = j < hd;
#pragma unroll
            for (int e = 0; e < 8; ++e)  // first half: x * cos + (-y) * sin; second: x * cos + y * sin
              ov[e] = rope_mul_add<T>(xv[e], cv[e], first ? (uint16_t)(yv[e] ^ 0x8000u) : yv[e], sv[e]);
            dst = head < p.n_q ? p.q + ((b * p.n_q + head) * p.S + s) * d
                               : p.k + ((b * p.n_kv + (head - p.n_q)) * p.S + s) * d;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) ov[e] = xv[e];
            dst = p.v + ((b * p.n_kv + (head - p.n_q - p.n_kv)) * p.S + s) * d;
          }
          *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(ov);
        }
        __syncwarp();
        asm volatile("bar.sync 1, 256;" ::: "memory");  // tout is reused by the next owned tile
      }
    }
    if (!arrived) arrive_cluster();
    if (et == 0) FQKV_TRACE_POINT(16);
    (void)ok;
  }

  // ---------------------------------------------------------------- teardown
  // The cluster barrier completes once every thread of every CTA has arrived, i.e. once no
  // CTA will reach into another's shared memory again; only then may a CTA leave (and
  // free its TMEM: every thread's tcgen05.ld came before its arrival).
  cluster_wait_acquire_thread();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) FQKV_TRACE_END();
}

template <int MPAD, int NT>
auto kernel_ptr(bool bf16) {
  return bf16 ? pipe_decode_kernel<__nv_bfloat16, MPAD, NT> : pipe_decode_kernel<__half, MPAD, NT>;
}

using KernelFn = void (*)(CUtensorMap, PipeParams, int);

KernelFn pick_kernel(int mpad, int nt, bool bf16) {
  switch (nt) {
    case 1: return mpad == 16 ? kernel_ptr<16, 1>(bf16) : mpad == 32 ? kernel_ptr<32, 1>(bf16) : nullptr;
    case 2: return mpad == 16 ? kernel_ptr<16, 2>(bf16) : mpad == 32 ? kernel_ptr<32, 2>(bf16) : nullptr;
    case 3: return mpad == 16 ? kernel_ptr<16, 3>(bf16) : mpad == 32 ? kernel_ptr<32, 3>(bf16) : nullptr;
    case 4: return mpad == 16 ? kernel_ptr<16, 4>(bf16) : mpad == 32 ? kernel_ptr<32, 4>(bf16) : nullptr;
    case 5: return mpad == 16 ? kernel_ptr<16, 5>(bf16) : mpad == 32 ? kernel_ptr<32, 5>(bf16) : nullptr;
    default: return nullptr;
  }
}

cudaLaunchConfig_t base_config(const PipeConfig& c, int groups, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c.cluster, (unsigned)groups);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = c.smem;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)c.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// How many clusters of this configuration the device keeps resident at once (cached).
int max_active_clusters(const PipeConfig& c, int groups) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, c.mpad, c.nt, c.cluster, c.smem);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  KernelFn k = pick_kernel(c.mpad, c.nt, true);
  int n = 0;
  if (k && ensure_smem_attr(reinterpret_cast<const void*>(k), c.smem) == cudaSuccess) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = base_config(c, groups, attr);
    if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

constexpr size_t kSmemLimit = 232448;  // max dynamic shared memory per block on sm_100
constexpr size_t kMinSmem = 80 * 1024;  // more than a third of the SM's 228 KB

}  // namespace

size_t pipe_smem_bytes(const PipeConfig& c, int kb_total) {
  const int nkb_max = (kb_total + c.cluster - 1) / c.cluster;
  return 1024 + make_pipe_layout(c.stages, c.nt, c.mpad, nkb_max, c.cluster).total;
}

// Choose (tile rows per CTA, cluster size, ring depth) for M <= 32 rows: every cluster
// resident at once (cudaOccupancyMaxActiveClusters), the most SMs streaming, then the
// deepest ring that fits (at most `kMaxStages`: the ring is what the producer fills while
// the preceding grid runs).  FQKV_PIPE_NT / FQKV_PIPE_CLUSTER / FQKV_PIPE_STAGES restrict
// the search (tuning).
int pipe_pick_config(int M, int H, int N, int sm_count, PipeConfig* cfg) {
  const int mpad = M <= 16 ? 16 : M <= 32 ? 32 : 0;
  if (mpad == 0) return FQKV_ERR_SCHEDULE;
  static const int force_nt = env_int("FQKV_PIPE_NT", 0);
  static const int force_c = env_int("FQKV_PIPE_CLUSTER", 0);
  static const int force_s = env_int("FQKV_PIPE_STAGES", 0);
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, std::pair<int, PipeConfig>> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, mpad, H, N, sm_count);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      if (it->second.first == 0) *cfg = it->second.second;
      return it->second.first;
    }
  }
  constexpr int kMaxStages = 16;
  PipeConfig best{};
  long best_score = -1;
  const int KB = (H + kKBlock - 1) / kKBlock;
  for (int nt = 1; nt <= kMaxNT; ++nt) {
    if (force_nt && nt != force_nt) continue;
    const int groups = (N + nt * kTileRows - 1) / (nt * kTileRows);
    for (int cl = 1; cl <= kMaxCluster && cl <= KB; ++cl) {
      if (force_c && cl != force_c) continue;
      if ((KB + cl - 1) / cl * 8 > kGainChunks * kNormThreads) continue;  // gain slice held in registers
      if ((long)groups * cl > sm_count) continue;
      for (int st = kMaxStages; st >= 2; --st) {
        if (force_s && st != force_s) continue;
        PipeConfig t{mpad, nt, st, cl, 0};
        t.smem = pipe_smem_bytes(t, KB);
        if (t.smem > kSmemLimit) continue;
        // At most two CTAs of these kernels share an SM (TMEM: two allocations of at most 256
        // columns fit the SM's 512, so no allocation ever waits on another CTA of the launch).
        t.smem = std::max(t.smem, kMinSmem);
        if (max_active_clusters(t, groups) < groups) continue;  // would need a second wave
        const long score = (long)groups * cl * 64 + st;
        if (score > best_score) {
          best_score = score;
          best = t;
        }
        break;  // deepest ring that fits for this (nt, cl)
      }
    }
  }
  const int rc = best_score < 0 ? FQKV_ERR_SCHEDULE : 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = std::make_pair(rc, best);
  }
  if (rc == 0) *cfg = best;
  return rc;
}

cudaError_t launch_pipe(const PipeConfig& c, const CUtensorMap& tmW, const PipeParams& p, bool bf16, bool pdl,
                        cudaStream_t stream) {
  KernelFn k = pick_kernel(c.mpad, c.nt, bf16);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(k), c.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  const int groups = (p.N + c.nt * kTileRows - 1) / (c.nt * kTileRows);
  cudaLaunchConfig_t cfg = base_config(c, groups, attr);
  cfg.stream = stream;
  if (pdl) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  // Weight stages issued before the activation loads once the preceding grid has completed
  // (before that, the whole ring): FQKV_PIPE_PRE, default 2.
  static const int pre_env = env_int("FQKV_PIPE_PRE", 0);
  PipeParams q = p;
  q.pre_stages = pre_env > 0 ? pre_env : 2;
  return cudaLaunchKernelEx(&cfg, k, tmW, q, c.stages);
}

}  // namespace fqkv
