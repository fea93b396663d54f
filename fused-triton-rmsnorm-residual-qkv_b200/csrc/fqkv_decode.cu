// fqkv_decode.cu -- the fused small-M (decode) kernel: residual add, RMSNorm and the
// projection in one launch, swap-AB tcgen05 GEMM with K split across a cluster.
//
// Decode (M = tokens <= 64) reads the whole weight once and little else, so it is
// HBM-bound.  The kernel computes D^T = W * normed^T: a 128-row tile of the packed
// weight is the MMA's A operand (M = 128) and the M tokens, padded to MPAD, are its
// N operand, so the output features fill the tensor core's M dimension.
//
// Grid = (C, n_tiles), cluster = (C, 1, 1).  CTA `rank` of a cluster owns the
// contiguous K slice [kb0, kb1) (64-element k-blocks) of n-tile blockIdx.y (NT x 128
// weight rows, NT = 1 .. 5).  Warp roles (320 threads):
//   warp 0     TMA producer: streams the CTA's weight slice through a STAGES-deep
//              ring of 128B-swizzled tiles (no multicast).
//   warp 1     TMEM allocator and single-thread MMA issuer (tcgen05.mma kind::f16,
//              fp32 accumulators in TMEM, tcgen05.commit frees ring stages).
//   warps 2-9  norm + epilogue.  Read x (+ residual) for the slice, form
//              h = dtype(x + r) (bit-exact, baseline.py:48), write the updated residual
//              (n-tile 0 only), keep h in shared memory in the UMMA operand layout,
//              exchange per-row partial sums of squares across the cluster through
//              DSMEM, then normalise in place: dtype((h * rstd) * g) (baseline.py:59-62).
//              The normalised activations never leave shared memory.
//              Epilogue: TMEM -> registers -> shared memory; each CTA bulk-copies
//              the slice of its partial tile that rank o owns into rank o's idle buffers
//              (cp.async.bulk shared::cta -> shared::cluster), and each owner sums the C
//              partials of its slice in rank order (deterministic) and stores it.
// F8 variant (e4m3 weights with an fp32 scale per weight row): the ring holds 128-byte e4m3
// rows (two k-blocks) that the MMA reads as they land (tcgen05.mma kind::f8f6f4, e4m3 x e4m3,
// fp32 accumulate).  The normalised activations, formed exactly as on the 16-bit path, are
// scaled per token by a power of two and split exactly into e4m3 terms (two for bf16, three
// for fp16), so the k-summed products equal those of the 16-bit values; the epilogue undoes
// the power of two and multiplies by the weight-row scale.
// The host sizes (NT, C, STAGES) so that all clusters are resident at once
// (cudaOccupancyMaxActiveClusters): a second wave would double the time.
// Every wait is bounded (fqkv_device.cuh); after a timeout the kernel drains its own
// TMA loads and MMAs, frees TMEM and returns with the status word set.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <map>
#include <tuple>
#include <type_traits>

#include "fqkv_kernels.cuh"

namespace fqkv {
namespace {

constexpr int kNormWarps = 8;                  // warps 2 .. 9: norm, then epilogue
constexpr int kNormThreads = kNormWarps * 32;
constexpr int kThreads = 64 + kNormThreads;
// Named barriers (barrier 0 is __syncthreads; 1 is the norm warps' own, 256 threads).
constexpr int kSetupBar = 2;      // set-up of warps 0 and 1 -> the norm warps
constexpr int kSetupPairBar = 3;  // thread 0's mbarrier initialisation -> the MMA warp
static_assert(kThreads == kDecodeThreads, "fqkv_kernels.cuh states the decode kernel's block size");
// Portable cluster sizes only: 16-CTA clusters (non-portable) were measured slower on the
// small per-GPU weight slices that could use them (N = 768: 7.70 against 7.37 us at C = 8).
constexpr int kMaxCluster = 8;
constexpr int kTileRows = 128;      // rows of W per MMA (UMMA M)
constexpr int kKBlock = 64;         // K elements per stage (128 bytes of 16-bit data)
constexpr int kWTileBytes = kTileRows * 128;
// e4m3 weights: a ring tile is 128 rows of 128 one-byte elements (two 64-deep k-blocks, one
// full 128-byte line per row), as many bytes as a 16-bit tile.  The activations' e4m3 terms
// take one MPAD x 128-byte region each per two k-blocks.
constexpr int kF8Batch = 8;                   // e4m3 weights: 16-byte chunks per lane and row in pass 2
constexpr int kF8Max = kF8Batch * 32 / 8;     // k-blocks of one CTA's K slice at most (pass 2 in registers)
constexpr int kF8SpreadPer = kF8Max * 8 / 64;  // e4m3, spread pass 2: chunks per thread at most (>= 64 per row)
__host__ __device__ constexpr int f8_terms(bool bf16) { return decode_f8_terms(bf16); }
constexpr int kLoadBatch = 4;       // 16-byte chunks per lane and row loaded before any is used
constexpr int kGridBatch = 8;       // grid variant: 16-byte chunks per thread loaded before any is used
constexpr int kGainChunks = 2;      // gain chunks per thread: K slices up to 2 * 256 * 8 elements
// Up to this many rows (cluster kernel, MPAD = 16, 16-bit or e4m3 weights), the norm phase
// spreads each row's chunks over several norm warps instead of giving each warp whole rows.
constexpr int kSpreadMaxM = 4;
static_assert(kNormWarps <= 16, "the spread norm phase's per-warp row sums fit rstd_s");
// log2 of the norm threads per row in the spread norm phase: all 256 for one row, 128 for
// two, 64 for three or four (a whole number of warps per row).
__host__ __device__ constexpr int spread_shift(int M) { return M == 1 ? 8 : M == 2 ? 7 : 6; }

struct Layout {
  uint32_t ring, stage_bytes, normed, gain, red, rowp, rstd, rscale, recvd, bars, tmem_slot, total;
};

// Receive slots of the cluster epilogue: in the ring after the partial tile (0), in the
// normalised-activation buffer (1), or in a region of their own (2).  In the first two the
// slots alias buffers a peer may still be using, so the cluster agrees that every CTA's MMAs
// have retired before any copy; a region of its own takes copies at any time.
constexpr int kRecvRing = 0, kRecvNormed = 1, kRecvOwn = kDecodeRecvOwn;
__host__ __device__ constexpr uint32_t recv_own_bytes(int nt, int mpad, int cluster) {
  // C slots of at most 32 * ceil(nt * mpad / C) quads (shares of whole 128-row blocks)
  return (uint32_t)(nt * mpad + cluster) * 128 * 4;
}

// f8 (the e4m3 terms of each activation, 0 for 16-bit weights): the ring holds e4m3 tiles
// (128-byte rows of two k-blocks, 128-byte swizzle); the activation buffer holds f8 regions
// of mpad x 128 bytes per two k-blocks (at least the 16-bit buffer the norm's first pass
// fills).
__host__ __device__ inline Layout make_layout(int stages, int nt, int mpad, int nkb_max, int f8, int recv_mode,
                                              int cluster) {
  Layout L;
  L.stage_bytes = nt * kWTileBytes;
  L.ring = 0;
  L.normed = L.ring + stages * L.stage_bytes;  // 1024-aligned: stages are multiples of 16 KB
  const int act_regions = f8 ? (nkb_max + 1) / 2 * f8 : nkb_max;
  L.gain = L.normed + (uint32_t)act_regions * mpad * 128;  // [nkb_max * 64] fp32 gain slice
  L.red = L.gain + (uint32_t)nkb_max * kKBlock * 4;  // [max(C, norm warps)][mpad] floats
  L.rowp = L.red + (uint32_t)(cluster > kNormWarps ? cluster : kNormWarps) * mpad * 4;  // [mpad] floats
  L.rstd = L.rowp + mpad * 4;                         // [mpad] floats
  L.rscale = L.rstd + mpad * 4;                       // f8: [mpad] 2^-s of each token's terms
  L.recvd = (L.rscale + mpad * 4 + 15) & ~15u;        // kRecvOwn: the C receive slots
  L.bars = (L.recvd + (recv_mode == kRecvOwn ? recv_own_bytes(nt, mpad, cluster) : 0u) + 7) & ~7u;
  // bars: full[S], empty[S], accum, normed, sum, part, acts, recv
  L.tmem_slot = L.bars + (2 * stages + 6) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

// dtype(dtype(a * c) + dtype(b * s)): PyTorch's a * c + b * s on 16-bit tensors, the rounding
// sequence of the separate rotary split (fqkv_rope.cu).
template <typename T>
__device__ __forceinline__ uint16_t rope_mul_add(uint16_t a, uint16_t c, uint16_t b, uint16_t s) {
  const uint16_t x = Elem<T>::from_f(__fmul_rn(Elem<T>::to_f(a), Elem<T>::to_f(c)));
  const uint16_t y = Elem<T>::from_f(__fmul_rn(Elem<T>::to_f(b), Elem<T>::to_f(s)));
  return Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(x), Elem<T>::to_f(y)));
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32u : cols <= 64 ? 64u : cols <= 128 ? 128u : cols <= 256 ? 256u : 512u;
}

template <typename T, int MPAD, int NT, bool F8, bool GRID, bool SPREAD>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmW, const DecodeParams p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  FQKV_TRACE_DECL
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = make_layout(stages, NT, MPAD, p.nkb_max, F8 ? f8_terms(std::is_same<T, __nv_bfloat16>::value) : 0,
                               p.recv_in_normed, (int)gridDim.x);
  uint8_t* ring = smem + L.ring;
  uint8_t* normed = smem + L.normed;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* rowp = reinterpret_cast<float*>(smem + L.rowp);
  float* rstd_s = reinterpret_cast<float*>(smem + L.rstd);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + stages;
  uint64_t* accum_bar = empty + stages;
  uint64_t* normed_bar = accum_bar + 1;
  uint64_t* sum_bar = accum_bar + 2;
  uint64_t* part_bar = accum_bar + 3;  // every CTA of the cluster has written its partial tile
  uint64_t* acts_bar = accum_bar + 4;  // the norm warps have issued their activation loads
  uint64_t* recv_bar = accum_bar + 5;  // the peers' slices of this CTA's share have landed
  float* rscale = reinterpret_cast<float*>(smem + L.rscale);
  // The gain slice as two arrays of 16-byte halves (elements 0-3 and 4-7 of each 8-element
  // chunk), so that a warp's 16-byte loads of consecutive chunks hit every bank once.
  float4* gain_lo = reinterpret_cast<float4*>(smem + L.gain);
  float4* gain_hi = gain_lo + p.nkb_max * (kKBlock / 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  // The epilogue reuses buffers the MMAs no longer need: this CTA's partial tile
  // [MPAD][NT][128] floats at the start of the ring, and C receive slots for the peers'
  // slices of the part of the tile this CTA reduces, in the normalised-activation buffer
  // when they fit there (else after the partial tile in the ring).
  float* part = reinterpret_cast<float*>(ring);
  constexpr uint32_t kPartBytes = NT * MPAD * kTileRows * 4;
  uint8_t* recv = p.recv_in_normed == kRecvNormed ? normed
                 : p.recv_in_normed == kRecvOwn  ? smem + L.recvd
                                                 : ring + kPartBytes;
  const bool recv_own = p.recv_in_normed == kRecvOwn;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // C CTAs split K: the CTAs of a cluster, or (GRID) blockIdx.x of a row of independent CTAs.
  const uint32_t C = gridDim.x;
  const uint32_t rank = GRID ? blockIdx.x : cluster_ctarank();
  static_assert(!(GRID && (F8 || MPAD != 16)), "the grid variant takes 16-bit weights and at most 16 rows");
  const int KB = p.kb_total;
  const int kb0 = decode_slice_begin((int)rank, (int)C, KB, F8), kb1 = decode_slice_begin((int)rank + 1, (int)C, KB, F8);
  const int nkb = kb1 - kb0;
  const int n_base = blockIdx.y * NT * kTileRows;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kTerms = F8 ? f8_terms(kBF16) : 1;  // e4m3: terms of each activation, stacked along N
  // Accumulators [0, NT * kTerms * MPAD): tile nt's term t in columns (nt * kTerms + t) * MPAD.
  constexpr uint32_t kTmemCols = tmem_cols_for(NT * kTerms * MPAD);
  constexpr int kBoxTiles = decode_box_tiles(NT);

  // The tile's partial sums are reduced in 16-byte quads (4 output features): quad
  // f = ((m * NT + nt) * 128 + row) / 4 for token m < M; rank o reduces [F(o), F(o+1)).
  // With the rotary split, shares are whole 128-row blocks (m, nt): a head's two halves stay
  // with one CTA.
  const bool rope = !F8 && !GRID && p.q != nullptr;  // the rotary split: 16-bit weights, cluster kernel
  const uint32_t total4 = (uint32_t)(NT * p.M * (kTileRows / 4));
  auto share = [&](uint32_t o) {
    return rope ? (o * (uint32_t)(NT * p.M)) / C * (kTileRows / 4) : (o * total4) / C;
  };
  const uint32_t slot_bytes = rope ? 16u * (kTileRows / 4) * ((NT * MPAD + C - 1) / C)
                                   : 16u * ((NT * MPAD * (kTileRows / 4) + C - 1) / C);

  // ---------------------------------------------------------------- setup
  FQKV_TRACE_BEGIN();
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_bar, 1);
    mbar_init(normed_bar, 1);
    mbar_init(sum_bar, 1);      // local arrive + C * MPAD * 4 bytes of st.async from the cluster
    mbar_init(part_bar, C);     // one (relaxed, fenced) arrive per CTA of the cluster
    mbar_init(acts_bar, 1);
    mbar_init(recv_bar, 1);     // local arrive + the peers' bulk copies (complete_tx)
    fence_mbarrier_init_cluster();
    // This CTA expects C * MPAD row sums (4 bytes each) from the cluster's st.async writes,
    // and later C - 1 bulk copies of its share of the tile; both are declared before the
    // CTA's first cluster arrival, so no peer's write can come first.
    if (!GRID) {
      mbar_arrive_expect_tx_cluster(sum_bar, C * MPAD * 4);
      mbar_arrive_expect_tx_cluster(recv_bar, (C - 1) * 16u * (share(rank + 1) - share(rank)));
    }
    FQKV_TRACE_POINT(17);
  }
  const int nstage = F8 ? (nkb + 1) / 2 : nkb;  // e4m3: a ring stage holds two k-blocks
  auto issue_stage = [&](int i, int s, uint64_t pol_w) {
    mbar_arrive_expect_tx(&full[s], L.stage_bytes);
    // A stage holds NT 128-row tiles: one box of NT x 128 rows for NT <= 2, else NT boxes
    // of 128 rows (a TMA box dimension is at most 256).
#pragma unroll
    for (int j = 0; j < NT; j += kBoxTiles)
      tma_load_2d_hint(ring + s * L.stage_bytes + j * kWTileBytes, &tmW, &full[s], (kb0 + (F8 ? 2 * i : i)) * kKBlock,
                       n_base + j * kTileRows, pol_w);
  };
  // Set-up without a block-wide barrier, so that no role waits for a set-up step it does not
  // need.  Named barrier kSetupPairBar: warp 0 (thread 0 initialised the mbarriers) arrives,
  // the MMA warp waits for it.  Named barrier kSetupBar: warps 0 and 1 arrive once the
  // mbarriers are initialised and TMEM is allocated; the norm warps wait for it only before
  // their first use of either (after their activation loads, which therefore start as soon as
  // the preceding grid has been released, even in a CTA that starts late).  The cluster
  // arrival publishes the barriers to the peers, and a thread waits for the whole cluster
  // only before its first access to a peer (the norm warps before the row-sum exchange; the
  // other warps before leaving), so that the weight stream and the activation loads do not
  // wait for the cluster's slowest CTA to be set up.
  uint32_t tmem_base = 0;
  if (warp == 0) {
    if (lane == 0) tma_prefetch_desc(&tmW);
    if (lane == 0) FQKV_TRACE_POINT(18);
    __syncwarp();
    named_bar_arrive(kSetupPairBar, 64);
    named_bar_arrive(kSetupBar, kThreads);
    cluster_arrive_release();
    if (lane == 0) pdl_launch_dependents();
    if (lane == 0) FQKV_TRACE_POINT(3);
  } else if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
    named_bar_sync(kSetupPairBar, 64);
    named_bar_arrive(kSetupBar, kThreads);
    tc_fence_after();
    cluster_arrive_release();
    tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
    if (lane == 0) FQKV_TRACE_POINT(21);
  } else {
    cluster_arrive_release();
  }

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // The weight does not depend on the preceding grid when the caller says so: start
      // streaming it before that grid has finished.  Only `pre` stages go out before the
      // norm warps have requested their activations, so those small, latency-critical
      // loads are not queued behind megabytes of weight in the memory system.
      if (!(p.flags & FQKV_FLAG_STATIC_WEIGHTS)) pdl_wait();
      const int pre = min(nstage, min(stages, p.pre_stages));
      const uint64_t pol_w = policy_evict_first();
      bool ok = true;
      int s = 0, round = 0, issued = 0;
      for (int i = 0; i < nstage; ++i) {
        if (i == pre) {
          ok = mbar_wait(acts_bar, 0);
          FQKV_TRACE_POINT(5);
        }
        if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1))) break;
        issue_stage(i, s, pol_w);
        if (i == 0) FQKV_TRACE_POINT(4);
        ++issued;
        if (++s == stages) {
          s = 0;
          ++round;
        }
      }
      FQKV_TRACE_POINT(6);
      // Before leaving, make sure none of this CTA's loads is still in flight: the last
      // `stages` loads are the only ones that can be (bounded waits).
      for (int j = max(0, issued - stages); j < issued; ++j) mbar_wait(&full[j % stages], (j / stages) & 1);
      (void)ok;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = F8 ? make_idesc_f8(kTileRows, kTerms * MPAD) : make_idesc_f16(kTileRows, MPAD, kBF16);
      bool ok = mbar_wait(normed_bar, 0);
      int s = 0, round = 0;
      for (int i = 0; i < nstage && ok; ++i) {
        if (!(ok = mbar_wait(&full[s], round & 1))) break;
        if (i == 0) FQKV_TRACE_POINT(11);
        if (i == nstage - 1) FQKV_TRACE_POINT(12);
        tc_fence_after();
        const uint32_t a_base = smem_u32(ring + s * L.stage_bytes);
        if (F8) {
          // e4m3: one stage is 128 K (two k-blocks); each 32-byte step is one MMA whose B
          // operand is the kTerms x MPAD rows of the terms' regions (contiguous), so the
          // terms' products land in kTerms column blocks of the tile's accumulator.
          const uint32_t b_base = smem_u32(normed + i * kTerms * MPAD * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = make_sw128_desc(b_base + kk * 32);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint64_t adesc = make_sw128_desc(a_base + nt * kWTileBytes + kk * 32);
              umma_f8(tmem_base + nt * kTerms * MPAD, adesc, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
        } else {
          const uint32_t b_base = smem_u32(normed + i * MPAD * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = make_sw128_desc(b_base + kk * 32);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint64_t adesc = make_sw128_desc(a_base + nt * kWTileBytes + kk * 32);
              umma_f16(tmem_base + nt * MPAD, adesc, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        umma_commit(&empty[s]);
        if (++s == stages) {
          s = 0;
          ++round;
        }
      }
      umma_commit(accum_bar);  // also on failure, so nobody waits for MMAs that never come
      mbar_wait(accum_bar, 0);  // all MMAs retired before TMEM is freed
    }
  } else {
    // ------------------------------------------------------------ norm + epilogue (warps 2..9)
    const int et = threadIdx.x - 64;  // 0 .. kNormThreads - 1
    bool ok = true;
    const int nw = warp - 2;
    const int nchunk = nkb * 8;  // 16-byte chunks per row of the slice
    const int64_t k_lo = (int64_t)kb0 * kKBlock;
    const bool static_w = (p.flags & FQKV_FLAG_STATIC_WEIGHTS) != 0;
    const bool write_res = p.rout != nullptr && blockIdx.y == 0;
    // The gain slice: loads go out now (into registers) and land in shared memory after
    // pass 1, so their latency overlaps that of the activations.  It is a weight: with
    // static weights it is read before the preceding grid has finished.
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
    // Warm L2 with this CTA's slice of x and the residual (one prefetch per 128-byte line)
    // while the preceding grid may still be running: a prefetch moves no data into
    // registers, and L2 is where a later write of that grid lands, so the loads after
    // pdl_wait still see every write.  Measured on B200 (Llama-3-8B, graph-timed): M = 16
    // 13.06 -> 12.89 us; at M = 1 it costs ~0.1 us, so single rows skip it.
    if (p.M > 1) {
      const int nline = (nchunk + 7) >> 3;  // 128-byte lines of a row's slice
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
    // Pass 1: warp nw takes rows nw, nw + 8, nw + 16, ... two at a time; each lane issues
    // up to kLoadBatch chunk loads of x (and r) per row before consuming any, so a pair of
    // rows costs one memory latency (M = 16: one pair per warp).  When that is all of the
    // warp's work (MPAD = 16 and at most 32 * kLoadBatch chunks per row), h also stays in
    // registers for pass 2.
    // SPREAD (M <= kSpreadMaxM, cluster kernel): each row's chunks over 256 / M (rounded down to
    // a power of two) threads, so they do not all fall to one warp.
    constexpr bool spread = SPREAD;
    static_assert(!SPREAD || (!GRID && MPAD == 16), "the spread norm phase: cluster kernel, MPAD 16");
    const bool h_in_regs = !GRID && !spread && MPAD == 2 * kNormWarps && nchunk <= 32 * kLoadBatch;
    uint4 hkeep[2][kLoadBatch];
    if constexpr (GRID) {
      // Whole rows: every CTA forms h = x + r over the entire row and its sum of squares
      // itself, chunk j of row m in thread j % 256 and in the same order in every CTA, so
      // all CTAs of a tile group get the same rstd and none waits for another.  h of this
      // CTA's K slice goes into the operand buffer; tile group 0 writes the updated
      // residual of its slices.  Rows M .. 15 of the buffer are left as they are: they only
      // reach accumulator columns that are never read.
      const int row_chunks = p.H >> 3;  // H % 8 == 0 on this path
      const int cpt = (row_chunks + kNormThreads - 1) / kNormThreads;  // chunks per thread and row
      const int units = p.M * cpt;
      const int j_lo = (int)(k_lo >> 3);
      uint64_t ssg[kGridMaxM];
#pragma unroll
      for (int m = 0; m < kGridMaxM; ++m) ssg[m] = 0ull;
      for (int u0 = 0; u0 < units; u0 += kGridBatch) {
        uint4 xv[kGridBatch], rv[kGridBatch];
#pragma unroll
        for (int b = 0; b < kGridBatch; ++b) {
          const int u = u0 + b, m = u / cpt, j = et + kNormThreads * (u - m * cpt);
          xv[b] = rv[b] = make_uint4(0, 0, 0, 0);
          if (u < units && j < row_chunks) {
            xv[b] = __ldg(reinterpret_cast<const uint4*>(p.x + (int64_t)m * p.ldx + (int64_t)j * 8));
            if (p.r) rv[b] = __ldg(reinterpret_cast<const uint4*>(p.r + (int64_t)m * p.ldr + (int64_t)j * 8));
          }
        }
#pragma unroll
        for (int b = 0; b < kGridBatch; ++b) {
          const int u = u0 + b, m = u / cpt, j = et + kNormThreads * (u - m * cpt);  // m: same in every thread
          if (u >= units) break;
          const uint4 hv = p.r ? add8_rn<T>(xv[b], rv[b]) : xv[b];
#pragma unroll
          for (int mm = 0; mm < kGridMaxM; ++mm)
            if (mm == m) ssg[mm] = sumsq8_f2<T>(hv, ssg[mm]);
          const int js = j - j_lo;  // chunk within this CTA's slice
          if (j < row_chunks && js >= 0 && js < nchunk) {
            *reinterpret_cast<uint4*>(normed + (js >> 3) * (MPAD * 128) + sw128_offset(m, js & 7)) = hv;
            if (write_res) *reinterpret_cast<uint4*>(p.rout + (int64_t)m * p.ldro + (int64_t)j * 8) = hv;
          }
        }
      }
      // The slice's chunks past the end of the row (H % 64 != 0) meet the weight map's
      // zero fill; they must hold finite values, so zeros.
      for (int t = et; t < p.M * nchunk; t += kNormThreads) {
        const int m = t / nchunk, js = t - m * nchunk;
        if (j_lo + js >= row_chunks)
          *reinterpret_cast<uint4*>(normed + (js >> 3) * (MPAD * 128) + sw128_offset(m, js & 7)) =
              make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int m = 0; m < kGridMaxM; ++m) {
        if (m < p.M) {
          float lo, hi;
          f2_unpack(ssg[m], lo, hi);
          float ss = lo + hi;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (lane == 0) red[nw * MPAD + m] = ss;
        }
      }
    } else if (spread) {
      // Row m = et / tpr, its chunks j = et % tpr (+ tpr, ...): 256, 128 or 64 threads per row
      // for M = 1, 2 or 3-4.  Each warp serves one row; the warps' sums of squares go to
      // rstd_s[warp] (free until the rows' rstd is formed), and the cluster exchange adds a
      // row's warps in order.
      const int shift = spread_shift(p.M), tpr = 1 << shift;
      const int m = et >> shift, jj = et & (tpr - 1);
      const bool row_live = m < p.M;
      uint64_t ssp = 0ull;
      for (int j0 = jj; j0 < nchunk; j0 += 2 * tpr) {
        uint4 xv[2], rv[2];
  #pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int j = j0 + tpr * b;
          const int64_t k = k_lo + (int64_t)j * 8;
          xv[b] = rv[b] = make_uint4(0, 0, 0, 0);
          if (row_live && j < nchunk && k < p.H) {
            xv[b] = __ldg(reinterpret_cast<const uint4*>(p.x + (int64_t)m * p.ldx + k));
            if (p.r) rv[b] = __ldg(reinterpret_cast<const uint4*>(p.r + (int64_t)m * p.ldr + k));
          }
        }
  #pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int j = j0 + tpr * b;
          const int64_t k = k_lo + (int64_t)j * 8;
          if (row_live && j < nchunk) {  // chunks past the end of the row hold zeros
            const uint4 hv = p.r ? add8_rn<T>(xv[b], rv[b]) : xv[b];
            ssp = sumsq8_f2<T>(hv, ssp);
            if (write_res && k < p.H) *reinterpret_cast<uint4*>(p.rout + (int64_t)m * p.ldro + k) = hv;
            *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) = hv;
          }
        }
      }
      float lo, hi;
      f2_unpack(ssp, lo, hi);
      float ss = lo + hi;
  #pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rstd_s[nw] = ss;
    } else {
      for (int m0 = nw; m0 < MPAD; m0 += 2 * kNormWarps) {
        uint64_t ss2[2] = {0ull, 0ull};  // fp32 pairs: even / odd elements
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
            // Branch-free over the batch (predicated stores only), so the chunks interleave:
            // x and r are zero where a chunk is out of range, so h is zero and adds nothing.
  #pragma unroll
            for (int b = 0; b < kLoadBatch; ++b) {
              const int j = j0 + lane + 32 * b;
              const int64_t k = k_lo + (int64_t)j * 8;
              const uint4 hv = p.r ? add8_rn<T>(xv[q2][b], rv[q2][b]) : xv[q2][b];
              ss2[q2] = sumsq8_f2<T>(hv, ss2[q2]);
              if (write_res && live && j < nchunk && k < p.H)
                *reinterpret_cast<uint4*>(p.rout + (int64_t)m * p.ldro + k) = hv;
              hkeep[q2][b] = hv;
              if (live && j < nchunk)
                *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) = hv;
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
    }
#pragma unroll
    for (int i = 0; i < kGainChunks; ++i) {
      const int j = et + kNormThreads * i;
      if (j < nchunk) {
        float4 gv[2];
        gain_raw_to_f32(p.gdt, graw[i], gv);
        gain_lo[j] = gv[0];
        gain_hi[j] = gv[1];
      }
    }
    // All norm warps, and the set-up of warps 0 and 1 (mbarriers initialised, TMEM allocated).
    named_bar_sync(kSetupBar, kThreads);
    tc_fence_after();
    tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
    // Every activation load has returned: the producer may now fill the whole ring.
    if (et == 0) mbar_arrive(acts_bar);
    if (et == 0) FQKV_TRACE_POINT(8);
    cluster_wait_acquire();  // every CTA of the cluster has initialised its barriers
    if constexpr (GRID) {
      // Whole-row sums: the eight warps' shares, added in warp order.
      for (int m = et; m < p.M; m += kNormThreads) {
        float tot = 0.f;
        for (int w = 0; w < kNormWarps; ++w) tot += red[w * MPAD + m];
        rstd_s[m] = row_rstd(tot, p.H, p.eps);
      }
    } else {
      // Publish this CTA's per-row partial sums into slot `rank` of every CTA: each st.async
      // counts its 4 bytes on the receiving CTA's sum_bar.
      if (warp == 2) {
        float part_m = 0.f;  // spread: this lane's row (m = lane < M), its warps' sums in order
        if (spread && lane < p.M) {
          const int wpr = 1 << (spread_shift(p.M) - 5);  // warps per row
          for (int w = lane * wpr; w < (lane + 1) * wpr; ++w) part_m += rstd_s[w];
        }
        for (uint32_t c = 0; c < C; ++c) {
          const uint32_t bar_c = mapa_shared(smem_u32(sum_bar), c);
          for (int m = lane; m < MPAD; m += 32)
            st_async_f32(mapa_shared(smem_u32(&red[rank * MPAD + m]), c), spread ? part_m : rowp[m], bar_c);
        }
        if constexpr (SPREAD) __syncwarp();  // every lane has read the per-warp sums before rstd_s is overwritten
      }
      ok = mbar_wait<true>(sum_bar, 0);
      for (int m = et; m < MPAD; m += kNormThreads) {
        float tot = 0.f;
        for (uint32_t c = 0; c < C; ++c) tot += red[c * MPAD + m];
        rstd_s[m] = row_rstd(tot, p.H, p.eps);
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (et == 0) FQKV_TRACE_POINT(9);
    // Pass 2: normalise, dtype((h * rstd) * g), over pass 1's rows and chunks; a lane's gain
    // pairs for its kLoadBatch chunks are loaded once and serve all its rows.
    auto load_g2 = [&](int j, uint64_t (&g2)[4]) {
      const ulonglong2 a = reinterpret_cast<const ulonglong2*>(gain_lo)[j];
      const ulonglong2 c = reinterpret_cast<const ulonglong2*>(gain_hi)[j];
      g2[0] = a.x;
      g2[1] = a.y;
      g2[2] = c.x;
      g2[3] = c.y;
    };
    if (F8) {
      // e4m3 weights: per token row (a warp takes pass 1's pairs), the normalised values --
      // exactly the 16-bit path's -- times 2^s, with 2^s putting the row's largest magnitude
      // in [128, 256), split exactly into kTerms e4m3 terms (each the rounding of what the
      // earlier ones left); 2^-s goes to the epilogue.  The terms of every 128 K (two
      // k-blocks) fill kTerms regions of MPAD x 128 bytes, zeros beyond the slice.  Each warp
      // reads all of its rows before writing them (in place).
      const int nchunk16 = (nchunk + 15) & ~15;  // 16-byte chunks rounded up to whole 128 K
      // chunk j of row m: 8 values at byte 8 (j % 16) of the row's 128-byte line in the
      // terms' regions (j / 16) * kTerms + t
      auto term_off = [&](int m, int j) {
        return (uint32_t)((j >> 4) * kTerms) * (MPAD * 128) + (uint32_t)m * 128u +
               ((((uint32_t)(j & 15) >> 1) ^ ((uint32_t)m & 7u)) << 4) + ((uint32_t)(j & 1) << 3);
      };
      // NB 16-byte chunks per lane and row; kRegs: h is still in registers from pass 1.
      auto pass2_f8 = [&](auto nb_c, auto regs_c) {
        constexpr int NB = decltype(nb_c)::value;
        constexpr bool kRegs = decltype(regs_c)::value;
        for (int mb = nw; mb < p.M; mb += 2 * kNormWarps) {  // pass 1's row pairs (register slot q2)
          // Rows mb and mb + 8 (live when < M; the padding rows' terms are never written: they
          // reach only accumulator columns that are never read), both at once.
          const bool live1 = mb + kNormWarps < p.M;
          uint64_t rs2[2];
          rs2[0] = f2_pack(rstd_s[mb], rstd_s[mb]);
          rs2[1] = live1 ? f2_pack(rstd_s[mb + kNormWarps], rstd_s[mb + kNormWarps]) : 0ull;
          uint4 o[2][NB];
          uint32_t mx2[2] = {0u, 0u};
  #pragma unroll
          for (int b = 0; b < NB; ++b) {
            o[0][b] = o[1][b] = make_uint4(0, 0, 0, 0);
            if (32 * b < nchunk) {  // warp-uniform
              const int j = lane + 32 * b;
              const bool in = j < nchunk && k_lo + (int64_t)j * 8 < p.H;
              uint64_t g2[4];
              load_g2(j < nchunk ? j : nchunk - 1, g2);  // clamped: always inside the gain slice
  #pragma unroll
              for (int q2 = 0; q2 < 2; ++q2) {
                if (q2 == 1 && !live1) continue;
                const int m0 = mb + kNormWarps * q2;
                uint4 hv = make_uint4(0, 0, 0, 0);
                if constexpr (kRegs)
                  hv = hkeep[q2][b];
                else if (in)
                  hv = *reinterpret_cast<const uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m0, j & 7));
                if (in) {
                  o[q2][b] = normalize8_f2<T>(hv, rs2[q2], g2);
                  mx2[q2] = absmax8_bits(o[q2][b], mx2[q2]);
                }
              }
            }
          }
          float up[2] = {0.f, 0.f};
  #pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            if (q2 == 1 && !live1) continue;
            const uint32_t mxb = __reduce_max_sync(0xffffffffu, max(mx2[q2] & 0xFFFFu, mx2[q2] >> 16));
            const float mx = Elem<T>::to_f((uint16_t)mxb);
            // mx in [2^e, 2^(e+1)): scale by 2^(7 - e).
            const int e = mx > 0.f ? (int)((__float_as_uint(mx) >> 23) & 0xFFu) - 127 : 7;
            const int sh = min(max(7 - e, -100), 100);
            up[q2] = __uint_as_float((uint32_t)(127 + sh) << 23);
            if (lane == 0) rscale[mb + kNormWarps * q2] = __uint_as_float((uint32_t)(127 - sh) << 23);
          }
          if (et == 0) FQKV_TRACE_POINT(19);
          __syncwarp();  // every lane has read its rows before any lane writes the terms over them
  #pragma unroll
          for (int b = 0; b < NB; ++b) {
            const int j = lane + 32 * b;
            if (32 * b < nchunk16 && j < nchunk16) {
  #pragma unroll
              for (int q2 = 0; q2 < 2; ++q2) {
                if (q2 == 1 && !live1) continue;
                const int m0 = mb + kNormWarps * q2;
                uint2 t8[kTerms];
                split_e4m3<T, kTerms>(o[q2][b], up[q2], t8);
  #pragma unroll
                for (int t = 0; t < kTerms; ++t)
                  *reinterpret_cast<uint2*>(normed + term_off(m0, j) + t * (MPAD * 128)) = t8[t];
              }
            }
          }
        }
      };
      if constexpr (SPREAD) {
        // Spread (as in pass 1: row et / tpr, chunks et % tpr + tpr * b): every thread
        // normalises its chunks into registers and takes their largest magnitude; the row's
        // warps meet in shared memory for the row's power of two, and only after that barrier,
        // when every h of the slice has been read, are the terms written over the buffer.
        const int shift = spread_shift(p.M), tpr = 1 << shift;
        const int m = et >> shift, jj = et & (tpr - 1);
        const bool row_live = m < p.M;
        const uint64_t rs2 = row_live ? f2_pack(rstd_s[m], rstd_s[m]) : 0ull;
        uint4 o[kF8SpreadPer];
        uint32_t mx = 0u;
  #pragma unroll
        for (int b = 0; b < kF8SpreadPer; ++b) {
          o[b] = make_uint4(0, 0, 0, 0);
          const int j = jj + tpr * b;
          if (row_live && j < nchunk && k_lo + (int64_t)j * 8 < p.H) {
            uint64_t g2[4];
            load_g2(j, g2);
            const uint4 hv = *reinterpret_cast<const uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7));
            o[b] = normalize8_f2<T>(hv, rs2, g2);
            mx = absmax8_bits(o[b], mx);
          }
        }
        uint32_t* wmax = reinterpret_cast<uint32_t*>(rowp);  // per-warp maxima (rowp is unused when spread)
        const uint32_t mxw = __reduce_max_sync(0xffffffffu, max(mx & 0xFFFFu, mx >> 16));
        if (lane == 0) wmax[nw] = mxw;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (row_live) {
          uint32_t mxb = 0u;
          const int wpr = 1 << (shift - 5);  // warps per row
          for (int w = m * wpr; w < (m + 1) * wpr; ++w) mxb = max(mxb, wmax[w]);
          const float mxf = Elem<T>::to_f((uint16_t)mxb);
          // mx in [2^e, 2^(e+1)): scale by 2^(7 - e).
          const int e = mxf > 0.f ? (int)((__float_as_uint(mxf) >> 23) & 0xFFu) - 127 : 7;
          const int sh = min(max(7 - e, -100), 100);
          const float up = __uint_as_float((uint32_t)(127 + sh) << 23);
          if (jj == 0) rscale[m] = __uint_as_float((uint32_t)(127 - sh) << 23);
          const int nchunk16 = (nchunk + 15) & ~15;  // the terms of whole 128 K, zeros beyond the slice
  #pragma unroll
          for (int b = 0; b < kF8SpreadPer; ++b) {
            const int j = jj + tpr * b;
            if (j < nchunk16) {
              uint2 t8[kTerms];
              split_e4m3<T, kTerms>(o[b], up, t8);
  #pragma unroll
              for (int t = 0; t < kTerms; ++t)
                *reinterpret_cast<uint2*>(normed + term_off(m, j) + t * (MPAD * 128)) = t8[t];
            }
          }
        }
      } else if (h_in_regs) {
        pass2_f8(std::integral_constant<int, kLoadBatch>{}, std::true_type{});
      } else {
        pass2_f8(std::integral_constant<int, kF8Batch>{}, std::false_type{});
      }
    } else if (spread) {
      // As in pass 1: row et / tpr, chunks et % tpr (+ tpr, ...); h from the operand buffer.
      const int shift = spread_shift(p.M), tpr = 1 << shift;
      const int m = et >> shift;
      if (m < p.M) {
        const uint64_t rs2 = f2_pack(rstd_s[m], rstd_s[m]);
        for (int j = et & (tpr - 1); j < nchunk; j += tpr) {
          if (k_lo + (int64_t)j * 8 >= p.H) continue;  // past the end of the row: stays zero
          uint64_t g2[4];
          load_g2(j, g2);
          uint4* dst = reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7));
          *dst = normalize8_f2<T>(*dst, rs2, g2);
        }
      }
    } else if (h_in_regs) {
      if (nw < p.M) {  // rows nw and nw + 8; padding rows are skipped (warp-uniform)
        const bool live1 = nw + kNormWarps < p.M;
        uint64_t rs2[2];
        rs2[0] = f2_pack(rstd_s[nw], rstd_s[nw]);
        rs2[1] = live1 ? f2_pack(rstd_s[nw + kNormWarps], rstd_s[nw + kNormWarps]) : 0ull;
#pragma unroll
        for (int b = 0; b < kLoadBatch; ++b) {
          if (32 * b >= nchunk) continue;  // warp-uniform
          const int j = lane + 32 * b;
          const bool in = j < nchunk && k_lo + (int64_t)j * 8 < p.H;
          uint64_t g2[4];
          load_g2(j < nchunk ? j : nchunk - 1, g2);  // clamped: always inside the gain slice
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            if (q2 == 1 && !live1) continue;
            const int m = nw + kNormWarps * q2;
            const uint4 o = normalize8_f2<T>(hkeep[q2][b], rs2[q2], g2);
            if (in) *reinterpret_cast<uint4*>(normed + (j >> 3) * (MPAD * 128) + sw128_offset(m, j & 7)) = o;
          }
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
    if (et == 0) FQKV_TRACE_POINT(20);
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    // FQKV_FLAG_TEST_WITHHOLD (tests of the failure path): no arrival, so the MMA thread's
    // bounded wait runs out; it then commits no MMA and the kernel winds down as usual.
    if (et == 0 && !(p.flags & FQKV_FLAG_TEST_WITHHOLD)) mbar_arrive(normed_bar);
    if (et == 0) FQKV_TRACE_POINT(10);

    // Rotary split: unit u of this CTA's share is 8 features (rows r8 .. r8 + 7 of local
    // block lb) of one token; a thread's first unit's cos / sin are loaded before the MMAs
    // finish, so that their latency stays out of the tail.
    struct RopeUnit {
      uint32_t lb;
      int r8, m, nn, head, j;
      int64_t b, sq;
    };
    auto rope_unit = [&](uint32_t u) {
      RopeUnit r;
      r.lb = u / (kTileRows / 8);
      r.r8 = (int)(u - r.lb * (kTileRows / 8)) * 8;
      const uint32_t mn = share(rank) / (kTileRows / 4) + r.lb;
      const int nt = (int)(mn % NT);
      r.m = (int)(mn / NT);
      r.nn = n_base + nt * kTileRows + r.r8;
      r.head = p.head_dim == 128 ? r.nn >> 7 : r.nn >> 6;  // head_dim is 64 or 128 on this path
      r.j = r.nn - r.head * p.head_dim;  // the 8 features stay in one half of a head
      r.b = (int64_t)((uint32_t)r.m / (uint32_t)p.S);  // M <= 32 tokens
      r.sq = r.m - r.b * p.S;
      return r;
    };
    const uint32_t rope_units = rope ? (share(rank + 1) - share(rank)) / (kTileRows / 4) * (kTileRows / 8) : 0u;
    uint4 cos0 = make_uint4(0, 0, 0, 0), sin0 = make_uint4(0, 0, 0, 0);
    if (!GRID && rope && (uint32_t)et < rope_units) {
      const RopeUnit r = rope_unit((uint32_t)et);
      if (r.nn < p.N && r.head < p.n_q + p.n_kv) {
        const int64_t cs = r.b * p.cs_batch_stride + r.sq * p.head_dim + r.j;
        cos0 = __ldg(reinterpret_cast<const uint4*>(p.cos + cs));
        sin0 = __ldg(reinterpret_cast<const uint4*>(p.sin + cs));
      }
    }
    ok = mbar_wait(accum_bar, 0) && ok;
    if (et == 0) FQKV_TRACE_POINT(13);
    tc_fence_after();
    const int q = warp & 3;             // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;   // the two warps of a quadrant split the 16-column chunks
    const int row = q * 32 + lane;
    // Quad f = ((m * NT + nt) * 128 + row) / 4 of the k-summed tile: four output features
    // of token m, rounded to the dtype and stored.
    const bool vec_store = (p.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 7) == 0;
    auto store_quad = [&](uint32_t f, float4 acc) {
      const int nl = (int)(f % (kTileRows / 4)) * 4;
      const uint32_t mn = f / (kTileRows / 4);
      const int nt = (int)(mn % NT), m = (int)(mn / NT);
      const int n = n_base + nt * kTileRows + nl;
      if (F8) {  // e4m3 weights: the row scale, once, on the k-summed value
        acc.x *= n < p.N ? p.wscale[n] : 0.f;
        acc.y *= n + 1 < p.N ? p.wscale[n + 1] : 0.f;
        acc.z *= n + 2 < p.N ? p.wscale[n + 2] : 0.f;
        acc.w *= n + 3 < p.N ? p.wscale[n + 3] : 0.f;
      }
      uint16_t* dst = p.out + (int64_t)m * p.ldo + n;
      if (vec_store && n + 3 < p.N) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(Elem<T>::from_f2(acc.x, acc.y), Elem<T>::from_f2(acc.z, acc.w));
      } else {
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < p.N) dst[e] = Elem<T>::from_f(a4[e]);
      }
    };
    if constexpr (GRID) {
      // Grid epilogue: this CTA's partial tile [m][nt][row] (tokens m < M) goes to its slot
      // in the workspace; the CTA that arrives last on the tile group's counter sums the C
      // slots in rank order (the result does not depend on arrival order), stores the tile
      // and puts the counter back to zero.  Nobody waits for another CTA.  A CTA whose
      // bounded waits gave up still arrives, so the counter stays consistent.
      const uint32_t grp = blockIdx.y;
      const int slot_floats = p.M * NT * kTileRows;
      float* slot = p.gpart + ((int64_t)grp * C + rank) * slot_floats;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if ((nt & 1) != half) continue;
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + nt * MPAD, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (e < p.M) slot[(e * NT + nt) * kTileRows + row] = __uint_as_float(v[e]);
      }
      tc_fence_before();
      __threadfence();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      volatile uint32_t* last_flag = tmem_slot + 1;
      if (et == 0) *last_flag = atomicAdd(p.gcnt + grp, 1) == (int)C - 1 ? 1u : 0u;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (et == 0) FQKV_TRACE_POINT(14);
      if (*last_flag) {
        __threadfence();
        const float4* slots4 = reinterpret_cast<const float4*>(p.gpart + (int64_t)grp * C * slot_floats);
        const uint32_t total4 = (uint32_t)(slot_floats / 4);
        for (uint32_t f = et; f < total4; f += kNormThreads) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (uint32_t c = 0; c < C; ++c) {
            const float4 v = __ldcg(slots4 + c * total4 + f);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
          }
          store_quad(f, acc);
        }
        if (et == 0) p.gcnt[grp] = 0;
      }
      if (et == 0) FQKV_TRACE_POINT(16);
      cluster_arrive_release_thread();  // the teardown's (one-CTA) cluster barrier
    } else {
      // Cluster epilogue: TMEM -> registers -> this CTA's partial tile in shared memory, laid
      // out [m][nt][row] so that every rank's share is one contiguous byte range.
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int c0 = 0; c0 < MPAD; c0 += 16) {
          if (((nt * (MPAD / 16) + c0 / 16) & 1) != half) continue;
          uint32_t v[kTerms][16];
#pragma unroll
          for (int t = 0; t < kTerms; ++t)
            tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (nt * kTerms + t) * MPAD + c0, v[t]);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            // e4m3: the terms' sums in term order, then the token's power of two undone (exact)
            float a = __uint_as_float(v[0][e]);
#pragma unroll
            for (int t = 1; t < kTerms; ++t) a += __uint_as_float(v[t][e]);
            part[((c0 + e) * NT + nt) * kTileRows + row] = F8 ? a * rscale[c0 + e] : a;
          }
        }
      }
      tc_fence_before();
      // The bulk copies read the partial tile through the async proxy.
      fence_proxy_async_smem();
      // One release per CTA: the CTA barrier orders every thread's partial-tile writes before
      // thread 0's cluster fence, which the relaxed remote arrives then publish.  An arrival
      // also says that this CTA's MMAs have retired, so its ring may receive the peers' slices.
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (!recv_own) {
        if (et == 0) {
          fence_acq_rel_cluster();
          for (uint32_t c = 0; c < C; ++c) mbar_arrive_remote_relaxed(mapa_shared(smem_u32(part_bar), c));
        }
        ok = mbar_wait<true>(part_bar, 0) && ok;
      }
      if (et == 0) FQKV_TRACE_POINT(14);
      // Lane c of warp 2 sends rank c's share of this CTA's partial tile to slot `rank` of
      // rank c's ring.
      if (warp == 2 && (uint32_t)lane < C && (uint32_t)lane != rank) {
        const uint32_t o = (uint32_t)lane, f0 = share(o), nb = 16u * (share(o + 1) - f0);
        if (nb > 0)
          bulk_copy_to_peer(mapa_shared(smem_u32(recv) + rank * slot_bytes, o), smem_u32(part) + 16u * f0, nb,
                            mapa_shared(smem_u32(recv_bar), o));
      }
      ok = mbar_wait<true>(recv_bar, 0) && ok;
      if (et == 0) FQKV_TRACE_POINT(15);
      // Every copy into this CTA has landed, so their sources have been read: this thread
      // makes no further access to a peer's shared memory, nor a peer to this CTA's.  The
      // barrier only has to order execution (the copies' data is tracked by their mbarriers).
      cluster_arrive_relaxed_thread();
      // Reduce this CTA's share: the C partials of each quad in rank order (deterministic).
      const uint32_t f0 = share(rank), f1 = share(rank + 1);
      const float4* part4 = reinterpret_cast<const float4*>(part);
      const float4* recv4 = reinterpret_cast<const float4*>(recv);
      // Rotary split: the rounded outputs of this CTA's blocks go to its own (unused) receive
      // slot, [local block][128] in the dtype, then out head-major.
      uint16_t* tout = reinterpret_cast<uint16_t*>(recv + rank * slot_bytes);
      for (uint32_t f = f0 + et; f < f1; f += kNormThreads) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t c = 0; c < C; ++c) {
          const float4 v = c == rank ? part4[f] : recv4[c * (slot_bytes / 16) + (f - f0)];
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        if (rope)
          *reinterpret_cast<uint2*>(tout + (f - f0) * 4) =
              make_uint2(Elem<T>::from_f2(acc.x, acc.y), Elem<T>::from_f2(acc.z, acc.w));
        else
          store_quad(f, acc);
      }
      if (rope) {
        // Head-major Q / K / V with the rotary embedding on Q and K, 8 features per thread
        // (the rounding sequence of fqkv_rope.cu: each product rounded to the dtype, their
        // fp32 sum rounded).
        __syncwarp();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const int d = p.head_dim, hd = d / 2;
        for (uint32_t u = et; u < rope_units; u += kNormThreads) {
          const RopeUnit ru = rope_unit(u);
          const int r8 = ru.r8, nn = ru.nn, head = ru.head, j = ru.j;
          const int64_t b = ru.b, sq = ru.sq;
          if (nn >= p.N) continue;
          const uint16_t* blk = tout + ru.lb * kTileRows;
          uint16_t xv[8], ov[8];
          *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(blk + r8);
          uint16_t* dst;
          if (head < p.n_q + p.n_kv) {
            uint16_t yv[8], cv[8], sv[8];
            *reinterpret_cast<uint4*>(yv) = *reinterpret_cast<const uint4*>(blk + (r8 ^ hd));  // other half
            if (u == (uint32_t)et) {  // loaded before the MMAs finished
              *reinterpret_cast<uint4*>(cv) = cos0;
              *reinterpret_cast<uint4*>(sv) = sin0;
            } else {
              const int64_t cs = b * p.cs_batch_stride + sq * d + j;
              *reinterpret_cast<uint4*>(cv) = __ldg(reinterpret_cast<const uint4*>(p.cos + cs));
              *reinterpret_cast<uint4*>(sv) = __ldg(reinterpret_cast<const uint4*>(p.sin + cs));
            }
            const bool first = j < hd;
#pragma unroll
            for (int e = 0; e < 8; ++e)  // first half: x * cos + (-y) * sin; second: x * cos + y * sin
              ov[e] = rope_mul_add<T>(xv[e], cv[e], first ? (uint16_t)(yv[e] ^ 0x8000u) : yv[e], sv[e]);
            dst = head < p.n_q ? p.q + ((b * p.n_q + head) * p.S + sq) * d
                               : p.k + ((b * p.n_kv + (head - p.n_q)) * p.S + sq) * d;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) ov[e] = xv[e];
            dst = p.v + ((b * p.n_kv + (head - p.n_q - p.n_kv)) * p.S + sq) * d;
          }
          *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(ov);
        }
      }
      if (et == 0) FQKV_TRACE_POINT(16);
    }
    (void)ok;
  }

  // ---------------------------------------------------------------- teardown
  if (warp < 2) {
    __syncwarp();
    cluster_wait_acquire_thread();  // the set-up phase of the cluster barrier
    tc_fence_before();
    cluster_arrive_relaxed_thread();
  }
  // No CTA leaves while a peer may still read its shared memory.
  cluster_wait_acquire_thread();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  FQKV_TRACE_END();
}

template <int MPAD, int NT, bool F8, bool GRID = false, bool SPREAD = false>
auto kernel_ptr(bool bf16) {
  return bf16 ? decode_kernel<__nv_bfloat16, MPAD, NT, F8, GRID, SPREAD>
              : decode_kernel<__half, MPAD, NT, F8, GRID, SPREAD>;
}

using KernelFn = void (*)(CUtensorMap, DecodeParams, int);

// Tile rows per CTA: 1 or 2 for every MPAD; 3 to 5 (wide weights: more SMs in one wave)
// for MPAD 16 and 32.
constexpr int kMaxNT = 5;

template <bool F8>
KernelFn pick_kernel_t(int mpad, int nt, bool bf16) {
  switch (nt) {
    case 1: return mpad == 16 ? kernel_ptr<16, 1, F8>(bf16) : mpad == 32 ? kernel_ptr<32, 1, F8>(bf16)
                 : mpad == 64 ? kernel_ptr<64, 1, F8>(bf16) : nullptr;
    case 2: return mpad == 16 ? kernel_ptr<16, 2, F8>(bf16) : mpad == 32 ? kernel_ptr<32, 2, F8>(bf16)
                 : mpad == 64 ? kernel_ptr<64, 2, F8>(bf16) : nullptr;
    case 3: return mpad == 16 ? kernel_ptr<16, 3, F8>(bf16) : mpad == 32 ? kernel_ptr<32, 3, F8>(bf16) : nullptr;
    case 4: return mpad == 16 ? kernel_ptr<16, 4, F8>(bf16) : mpad == 32 ? kernel_ptr<32, 4, F8>(bf16) : nullptr;
    case 5: return mpad == 16 ? kernel_ptr<16, 5, F8>(bf16) : mpad == 32 ? kernel_ptr<32, 5, F8>(bf16) : nullptr;
    default: return nullptr;
  }
}

KernelFn pick_kernel(int mpad, int nt, bool bf16, bool f8) {
  return f8 ? pick_kernel_t<true>(mpad, nt, bf16) : pick_kernel_t<false>(mpad, nt, bf16);
}

// The cluster kernel with the spread norm phase: MPAD 16, M <= kSpreadMaxM.
template <bool F8>
KernelFn pick_spread_kernel_t(int nt, bool bf16) {
  switch (nt) {
    case 1: return kernel_ptr<16, 1, F8, false, true>(bf16);
    case 2: return kernel_ptr<16, 2, F8, false, true>(bf16);
    case 3: return kernel_ptr<16, 3, F8, false, true>(bf16);
    case 4: return kernel_ptr<16, 4, F8, false, true>(bf16);
    case 5: return kernel_ptr<16, 5, F8, false, true>(bf16);
    default: return nullptr;
  }
}

KernelFn pick_spread_kernel(int nt, bool bf16, bool f8) {
  return f8 ? pick_spread_kernel_t<true>(nt, bf16) : pick_spread_kernel_t<false>(nt, bf16);
}

// Grid variant: 16-bit weights, MPAD 16, 1 to 5 tiles per CTA.
KernelFn pick_grid_kernel(int nt, bool bf16) {
  switch (nt) {
    case 1: return kernel_ptr<16, 1, false, true>(bf16);
    case 2: return kernel_ptr<16, 2, false, true>(bf16);
    case 3: return kernel_ptr<16, 3, false, true>(bf16);
    case 4: return kernel_ptr<16, 4, false, true>(bf16);
    case 5: return kernel_ptr<16, 5, false, true>(bf16);
    default: return nullptr;
  }
}

cudaLaunchConfig_t base_config(const DecodeConfig& c, int tiles, cudaLaunchAttribute* attr, int* na) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c.cluster, (unsigned)tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = c.smem;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c.grid ? 1u : (unsigned)c.cluster;  // grid variant: K split without a cluster
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  *na = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// How many clusters of this configuration the device keeps resident at once (cached).
int max_active_clusters(const DecodeConfig& c, int tiles) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, c.mpad, c.nt, c.cluster, c.smem, c.f8);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  KernelFn k = pick_kernel(c.mpad, c.nt, true, c.f8 != 0);
  int n = 0;
  if (k && ensure_smem_attr(reinterpret_cast<const void*>(k), c.smem) == cudaSuccess) {
    cudaLaunchAttribute attr[2];
    int na = 0;
    cudaLaunchConfig_t cfg = base_config(c, tiles, attr, &na);
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

}  // namespace

constexpr size_t kSmemLimit = 232448;  // max dynamic shared memory per block on sm_100

size_t decode_smem_bytes(const DecodeConfig& c, int kb_total) {
  const int nkb_max = decode_slice_max(c.cluster, kb_total, c.f8 != 0);
  return 1024 + make_layout(c.stages, c.nt, c.mpad, nkb_max, c.f8, c.recv_in_normed, c.cluster).total;
}

// Choose (tile rows, cluster size, ring depth).  Candidates must fit shared memory and
// have every cluster resident at once; among them the one using the most SMs wins (ties
// go to the deeper ring, then to the smaller cluster).
// FQKV_DECODE_NT / FQKV_DECODE_CLUSTER / FQKV_DECODE_STAGES restrict the search.
int decode_pick_config(int M, int H, int N, int sm_count, DecodeConfig* cfg, int f8) {
  const int mpad = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0;
  if (mpad == 0) return FQKV_ERR_SCHEDULE;
  // Tuning overrides, read once per process.
  static const int force_nt = env_int("FQKV_DECODE_NT", 0);
  static const int force_c = env_int("FQKV_DECODE_CLUSTER", 0);
  static const int force_s = env_int("FQKV_DECODE_STAGES", 0);
  // The epilogue's receive slots: a region of their own for 16-bit weights and up to 32 rows
  // (measured on B200, Llama-3-8B, graph-timed: M = 16 13.28 -> 12.72 us, M = 1 12.40 ->
  // 12.15 us against slots aliasing the ring / the activations, which need the cluster to
  // agree first that every CTA's MMAs have retired); FQKV_DECODE_RECV=1 forces the aliasing
  // slots (comparisons).
  static const int recv_mode_env = env_int("FQKV_DECODE_RECV", 0);
  // The search below queries occupancy for many candidates; its result is cached per
  // (device, MPAD, H, N, SM count, overrides), so a model's per-step calls skip it.
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int, int, int>, std::pair<int, DecodeConfig>> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, mpad, H, N, sm_count, force_nt, force_c, force_s * 4 + recv_mode_env,
                                   f8);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      if (it->second.first == 0) *cfg = it->second.second;
      return it->second.first;
    }
  }
  DecodeConfig best{};
  const int KB = (H + kKBlock - 1) / kKBlock;
  long best_score = -1;
  for (int nt = 1; nt <= kMaxNT; ++nt) {
    if (force_nt && nt != force_nt) continue;
    if (!pick_kernel(mpad, nt, true, f8 != 0)) continue;
    // TMEM: at most half an SM's 512 columns, so that two CTAs of a cluster placed on one SM
    // could always both allocate (each waits in tcgen05.alloc for the other otherwise).
    if (tmem_cols_for(nt * std::max(f8, 1) * mpad) > 256) continue;
    const int tile_bytes = kWTileBytes;  // one 128-row tile in the ring (e4m3: two k-blocks)
    const int tiles = (N + nt * kTileRows - 1) / (nt * kTileRows);
    for (int cl = 1; cl <= kMaxCluster && cl <= KB; ++cl) {
      if (force_c && cl != force_c) continue;
      if (f8 && cl > (KB + 1) / 2) continue;  // every CTA gets one e4m3 stage at least
      const int nkb_max = decode_slice_max(cl, KB, f8 != 0);
      if (nkb_max * 8 > kGainChunks * kNormThreads) continue;  // gain slice held in registers
      if (f8 && nkb_max > kF8Max) continue;  // e4m3: the slice's terms formed in registers
      // The epilogue's partial tile aliases the ring.  Its C receive slots get a region of
      // their own (16-bit weights, up to 32 rows) when that still leaves a ring of three
      // stages or more; otherwise they go into the normalised-activation buffer when they fit
      // there, else after the partial tile in the ring.
      const int part_bytes = nt * mpad * kTileRows * 4;
      const int recv_bytes = cl * 16 * ((nt * mpad * (kTileRows / 4) + cl - 1) / cl);
      const int alias_mode = recv_bytes <= nkb_max * mpad * 128 ? kRecvNormed : kRecvRing;
      // Deepest resident ring of a receive mode for this (nt, cl), or a config with stages 0.
      auto deepest = [&](int mode) {
        const int epi_bytes = part_bytes + (mode == kRecvRing ? recv_bytes : 0);
        const int min_stages = (epi_bytes + nt * tile_bytes - 1) / (nt * tile_bytes);
        for (int st = 16; st >= max(2, min_stages); --st) {
          if (force_s && st != force_s) continue;
          DecodeConfig t{mpad, nt, st, cl, 0, mode, f8};
          t.smem = decode_smem_bytes(t, KB);
          if (t.smem > kSmemLimit) continue;
          if (max_active_clusters(t, tiles) < tiles) continue;  // would need a second wave
          return t;
        }
        return DecodeConfig{mpad, nt, 0, cl, 0, mode, f8};
      };
      DecodeConfig t = deepest(alias_mode);
      if (recv_mode_env != 1 && mpad <= 32) {
        const DecodeConfig own = deepest(kRecvOwn);
        if (own.stages >= 3 || (own.stages > 0 && t.stages == 0)) t = own;
      }
      if (t.stages == 0) continue;
      // Most CTAs first; among equal counts, stages of two or more 128-row tiles (32 KB boxes
      // and up: one thread issues TMA boxes at a bounded rate, and 16 KB boxes stream well
      // below the copy peak), then the deepest ring.  Measured on B200 (Qwen2-7B, graph-timed,
      // both 108 CTAs): NT = 1, C = 3 10.48 / 13.30 us at M = 1 / 16, NT = 2, C = 6 9.47 / 10.52.
      const long score = ((long)tiles * cl * 2 + (nt >= 2 ? 1 : 0)) * 64 + t.stages;
      if (score > best_score) {
        best_score = score;
        best = t;
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

// The counters take a fixed region whatever the shape, so that one zero-filled workspace
// serves launches of different shapes: another shape's partial slots never overlap them.
int64_t decode_grid_counter_bytes() { return (int64_t)kGridMaxTiles * 4; }

// Counters, then the partial slots: groups x S x M x NT x 128 fp32, bounded by
// S <= kGridMaxSplit and groups x NT x 128 <= (ceil(N / 128) + kMaxNT) x 128.
int64_t decode_grid_workspace_bytes(int64_t M, int64_t N) {
  const int64_t tiles = (N + kTileRows - 1) / kTileRows;
  return decode_grid_counter_bytes() + (int64_t)kGridMaxSplit * (tiles + kMaxNT) * kTileRows * M * 4;
}

// Grid variant: NT tiles per CTA, S = cluster CTAs per tile group splitting K, S x groups
// <= SM count (one wave at one CTA per SM), S <= kGridMaxSplit.  The configuration with the
// fewest weight k-blocks per CTA wins (ties: more CTAs, then the deeper ring).
// FQKV_DECODE_NT / FQKV_DECODE_STAGES restrict the search as for the cluster kernel.
int decode_grid_pick_config(int M, int H, int N, int sm_count, DecodeConfig* cfg) {
  if (M < 1 || M > kGridMaxM || (N + kTileRows - 1) / kTileRows > kGridMaxTiles) return FQKV_ERR_SCHEDULE;
  static const int force_nt = env_int("FQKV_DECODE_NT", 0);
  static const int force_s = env_int("FQKV_DECODE_STAGES", 0);
  const int KB = (H + kKBlock - 1) / kKBlock;
  DecodeConfig best{};
  long best_cost = -1, best_ctas = 0;
  for (int nt = 1; nt <= kMaxNT; ++nt) {
    if (force_nt && nt != force_nt) continue;
    const int groups = (N + nt * kTileRows - 1) / (nt * kTileRows);
    if (groups > sm_count) continue;
    const int S = std::min(std::min(sm_count / groups, kGridMaxSplit), KB);
    const int nkb_max = (KB + S - 1) / S;
    if (nkb_max * 8 > kGainChunks * kNormThreads) continue;  // gain slice held in registers
    const long cost = (long)nt * nkb_max, ctas = (long)groups * S;
    for (int st = 16; st >= 2; --st) {
      if (force_s && st != force_s) continue;
      DecodeConfig t{16, nt, st, S, 0, 0, 0, 1};
      t.smem = decode_smem_bytes(t, KB);
      if (t.smem > kSmemLimit) continue;
      if (best_cost < 0 || cost < best_cost || (cost == best_cost && ctas > best_ctas)) {
        best_cost = cost;
        best_ctas = ctas;
        best = t;
      }
      break;  // deepest ring that fits for this NT
    }
  }
  if (best_cost < 0) return FQKV_ERR_SCHEDULE;
  *cfg = best;
  return 0;
}

cudaError_t launch_decode(const DecodeConfig& c, const CUtensorMap& tmW, const DecodeParams& p, bool bf16, bool pdl,
                          cudaStream_t stream) {
  // Rows up to kSpreadMaxM: the norm phase spread over the norm warps (measured on B200,
  // graph-timed: Llama-3-8B M = 1 / 4 11.99 / 12.08 -> 11.71 / 11.87 us, Llama-3-70B M = 1
  // 33.4 -> 30.8 us, e4m3 M = 1 9.86 -> 9.01 us).  The grid variant keeps one warp per row:
  // its pass 1 already reads whole rows over all threads, and the spread pass 2 was slower.
  const bool spread = !c.grid && c.mpad == 16 && p.M <= kSpreadMaxM;
  KernelFn k = c.grid ? pick_grid_kernel(c.nt, bf16)
               : spread ? pick_spread_kernel(c.nt, bf16, c.f8 != 0)
                        : pick_kernel(c.mpad, c.nt, bf16, c.f8 != 0);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(k), c.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  int na = 0;
  const int tiles = (p.N + c.nt * kTileRows - 1) / (c.nt * kTileRows);
  cudaLaunchConfig_t cfg = base_config(c, tiles, attr, &na);
  cfg.stream = stream;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.numAttrs = na;
  DecodeParams q = p;
  // Weight stages issued before the activation loads: 2 for the cluster kernel (swept 0-6
  // at NT = 2 on B200); about 64 KB for the grid variant, whose whole-row activation phase
  // is longer (graph-timed, Qwen2-7B shape, M = 1, NT = 1: 11.80 / 11.37 / 11.25 us with 2 /
  // 3 / 4 stages of 16 KB; at NT = 2, 2 stages beat 1).
  static const int pre_env = env_int("FQKV_DECODE_PRE", 0);  // read once per process
  const int grid_pre = std::max(1, (64 << 10) / (c.nt * kWTileBytes));
  q.pre_stages = pre_env > 0 ? pre_env : c.grid ? grid_pre : 2;
  q.recv_in_normed = c.recv_in_normed;
  return cudaLaunchKernelEx(&cfg, k, tmW, q, c.stages);
}

}  // namespace fqkv
