// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   D[m, n] = sum_k A[m, k] * B[n, k]        (both operands K-major, fp32 accumulate)
//
// One kernel template covers every GEMM-shaped op of the MLA-MoE model:
//   * MODE_DENSE   — persistent CTAs walk (m, n, batch) tiles; the TMEM
//                    accumulator is double buffered so the epilogue of tile i
//                    overlaps the main loop of tile i+1. Batched GEMMs (the
//                    per-head MLA absorb products) offset A rows, A/B K columns
//                    and D per batch index.
//   * MODE_SPLITK  — decode-shaped GEMMs (few tokens, weight-bandwidth bound):
//                    the K loop of one tile is split over `splits` independent
//                    CTAs with a short (4-stage) pipeline, so two fit per SM and
//                    the next kernel's CTAs can start early under PDL. (One SM's
//                    TMA stream tops out near 55 GB/s on these 128-byte rows, so
//                    an HBM-bound GEMM needs >100 SMs streaming at once.) Each
//                    CTA stores its fp32 partial with plain coalesced stores into
//                    a workspace slab; a wide split_reduce kernel sums the slabs
//                    into the output.
//   * MODE_GROUPED — MoE expert GEMMs: group g (an expert) owns A rows
//                    [g*M, g*M+M) and a device-side range of B rows (its sorted
//                    tokens); tile counts come from device memory, so the launch
//                    is CUDA-graph safe.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer + TMEM
// owner, warps 2..5 = epilogue (TMEM lane quarter = warp % 4).
// Operand tiles are 128-byte swizzled (64 bf16 of K per row); BLOCK_M = 128.
//
// The reference declares these products only as cuBLASLt "linear plans"
// (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:599-622)
// and the fused MoE entry points (same header :1046-1058); the math is written
// here from scratch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ll.cuh"
#include "pdl.h"

namespace sp {

// MODE_GROUPED_TM: token-major grouped GEMM for expert groups of prefill size: A is
// the expert-sorted tokens (M = a group's rows, 128 per tile), B the expert's weight
// rows (N), D row-major [rows, N] (or [rows, N / 2] with the fused SwiGLU: a tile's
// columns hold [64 gate | 64 up] features twice over, so each thread's token row
// pairs them from its own TMEM columns and writes 16 features with two 16-byte
// stores). The weight-major grouped mode keeps decode's swap-AB shape, whose
// transposed output is written two bytes at a time.
enum { MODE_DENSE = 0, MODE_SPLITK = 1, MODE_GROUPED = 2, MODE_GROUPED_TM = 3 };

struct GemmKParams {
  int M, N, K;
  int batch;
  int a_row0, a_batch_rows, a_k0, a_batch_k;
  int b_row0, b_batch_rows, b_k0, b_batch_k;
  void* D;
  long long ldd;
  long long d_batch_stride;
  int trans_out;
  int out_f32;
  int m_tiles, n_tiles, num_tiles;
  int splits;
  const int* grp_rows;   // [G+1]
  const int* grp_tiles;  // [G+1]
  int num_groups;
  int a_evict_first;  // A is a weight operand: stream it with evict_first and prefetch it before the PDL wait
  int sched_early;    // MODE_GROUPED: the tile schedule may be read before the PDL wait
  int swiglu;         // grouped: A rows are [64 gate | 64 up] per tile; write silu(gate) * up
  float* ws;          // split-K partial slabs: [splits][N][M] (trans_out) or [splits][M][N], fp32
  long long split_stride;
  // stream-K split (sk_ctas > 0): CTA c owns the flattened (tile, K-block) units
  // [c*T/G, (c+1)*T/G), G = sk_ctas; a tile's partials fill slab slots 0..nseg-1 and
  // the CTA finishing the tile zeroes slots nseg..sk_slots-1
  int sk_ctas, sk_slots;
  int* err;
  // Tensor parallelism over peer memory (LL tagged words, ll.cuh):
  //  * tp_rs: the epilogue sends fp32 partials of token n to rank n / tp_rows, slot
  //    (tp_rank * splits + split) of its reduce-scatter region [2][W*S][tp_rows][M];
  //  * tp_ag_flags: B is this rank's all-gather region [2][T][K] bf16 (the B tensor map
  //    covers both parity halves), written by the peers with plain stores; before a
  //    tile's first B load the producer waits (bounded, acquire) until the per-row
  //    flags of the tile's rows carry this layer's tag.
  unsigned long long tp_base[8];
  long long tp_rs_off;
  int tp_rs, tp_rank, tp_world, tp_rows;
  const unsigned long long* tp_ag_flags;  // [2][T] tags of this rank's all-gather region
  const int64_t* tp_epoch;
  int tp_layer, tp_layers_per_step;
  long long tp_budget;
  // expert-parallel combine epilogue (grouped): rows go to their source ranks' slots
  int ep_on;
  EpCombDev ep;
};

constexpr int BM = 128;
constexpr int BK = 64;

template <int BN, int MODE>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // split-K CTAs own only a few K blocks: a short pipeline keeps two CTAs per SM, so
  // under PDL the next kernel's CTAs can become resident beside them. (Eight stages for
  // decode-width split-K measured no faster: 16.6 vs 16.4 us at 64 x 9792 x 2048, so
  // bytes in flight do not bound it.)
  static constexpr int STAGES = MODE == MODE_SPLITK ? 4 : (BN >= 256 ? 4 : (BN >= 128 ? 6 : 8));
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int XBUF_BYTES = 64 * 17 * 4;  // SwiGLU exchange buffer (64 rows x 16 cols, padded)
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + XBUF_BYTES;
};

struct TileInfo {
  int a_row, a_k, b_row, b_k;
  int m_base, n_base;  // output coordinates of the tile origin
  int m_valid, n_valid;
  long long d_off;
};

template <int BN, int MODE>
SP_DEVI bool get_tile(const GemmKParams& p, int t, TileInfo& ti) {
  if (MODE == MODE_GROUPED_TM) {
    // n fastest: consecutive tiles reuse one token tile against the expert's weight tiles
    const int nt = t % p.n_tiles;
    const int q = t / p.n_tiles;  // global 128-row token tile
    int lo = 0, hi = p.num_groups;
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (__ldg(p.grp_tiles + mid) <= q) lo = mid; else hi = mid;
    }
    const int g = lo;
    const int mt = q - __ldg(p.grp_tiles + g);
    const int r0 = __ldg(p.grp_rows + g);
    const int r1 = __ldg(p.grp_rows + g + 1);
    ti.a_row = r0 + mt * BM;
    ti.a_k = p.a_k0;
    ti.b_row = p.b_row0 + g * p.b_batch_rows + nt * BN;
    ti.b_k = p.b_k0;
    ti.m_base = ti.a_row;
    ti.n_base = p.swiglu ? nt * (BN / 2) : nt * BN;
    ti.m_valid = min(BM, r1 - ti.a_row);
    ti.n_valid = min(BN, p.N - nt * BN);
    ti.d_off = 0;
    return ti.m_valid > 0;
  }
  if (MODE == MODE_GROUPED) {
    const int mt = t % p.m_tiles;
    const int q = t / p.m_tiles;
    // group = last g with grp_tiles[g] <= q
    int lo = 0, hi = p.num_groups;  // grp_tiles[lo] <= q < grp_tiles[hi]
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (__ldg(p.grp_tiles + mid) <= q) lo = mid; else hi = mid;
    }
    const int g = lo;
    const int nt = q - __ldg(p.grp_tiles + g);
    const int r0 = __ldg(p.grp_rows + g);
    const int r1 = __ldg(p.grp_rows + g + 1);
    ti.a_row = p.a_row0 + g * p.a_batch_rows + mt * BM;
    ti.a_k = p.a_k0;
    ti.b_row = r0 + nt * BN;
    ti.b_k = p.b_k0;
    ti.m_base = mt * BM;
    ti.n_base = ti.b_row;
    ti.m_valid = min(BM, p.M - mt * BM);
    ti.n_valid = min(BN, r1 - ti.b_row);
    ti.d_off = 0;
    return ti.n_valid > 0;
  } else {
    const int mt = t % p.m_tiles;
    const int r = t / p.m_tiles;
    const int nt = r % p.n_tiles;
    const int z = r / p.n_tiles;
    ti.a_row = p.a_row0 + z * p.a_batch_rows + mt * BM;
    ti.a_k = p.a_k0 + z * p.a_batch_k;
    ti.b_row = p.b_row0 + z * p.b_batch_rows + nt * BN;
    ti.b_k = p.b_k0 + z * p.b_batch_k;
    ti.m_base = mt * BM;
    ti.n_base = nt * BN;
    ti.m_valid = min(BM, p.M - mt * BM);
    ti.n_valid = min(BN, p.N - nt * BN);
    ti.d_off = (long long)z * p.d_batch_stride;
    return true;
  }
}

// CTA owning flattened unit w when W units are split over G CTAs.
SP_DEVI int sk_cta_of(long long w, long long W, int G) { return int(((w + 1) * G + W - 1) / W) - 1; }

// One item of a CTA's work: a tile, its K-block range [kb0, kb1), and (split-K) the
// slab slot of the partial and how many slots the tile's partials fill.
struct WorkItem {
  int tile, kb0, kb1, slot, nseg;
};

// The idx-th work item of this CTA; false past the last one.
template <int MODE>
SP_DEVI bool work_item(const GemmKParams& p, int num_tiles, int idx, WorkItem& w) {
  const int kbs = (p.K + BK - 1) / BK;
  if (MODE != MODE_SPLITK) {  // persistent: tiles blockIdx.x, + gridDim.x, ...
    const long long t = blockIdx.x + (long long)idx * gridDim.x;
    if (t >= num_tiles) return false;
    w.tile = int(t); w.kb0 = 0; w.kb1 = kbs; w.slot = 0; w.nseg = 1;
    return true;
  }
  if (p.sk_ctas == 0) {  // fixed split: CTA (tile, ks) owns K-block slice ks of one tile
    if (idx > 0) return false;
    const int ks = blockIdx.x % p.splits;
    w.tile = blockIdx.x / p.splits;
    w.kb0 = int((long long)kbs * ks / p.splits);
    w.kb1 = int((long long)kbs * (ks + 1) / p.splits);
    w.slot = ks;
    w.nseg = p.splits;
    return w.tile < num_tiles;
  }
  const long long T = (long long)num_tiles * kbs;
  const int G = p.sk_ctas, c = blockIdx.x;
  const long long u_end = T * (c + 1) / G;
  long long u = T * c / G;
  for (int i = 0; i < idx && u < u_end; ++i) u = min(u_end, (u / kbs + 1) * kbs);  // skip idx pieces
  if (u >= u_end) return false;
  const long long t = u / kbs;
  w.tile = int(t);
  w.kb0 = int(u - t * kbs);
  w.kb1 = int(min(u_end, (t + 1) * kbs) - t * kbs);
  const int cf = sk_cta_of(t * kbs, T, G), cl = sk_cta_of(t * kbs + kbs - 1, T, G);
  w.slot = c - cf;
  w.nseg = cl - cf + 1;
  return true;
}

template <int BN>
SP_DEVI void store_chunk(const GemmKParams& p, const TileInfo& ti, int m, int c0, const float (&v)[16]) {
  if (m >= ti.m_valid) return;
  const long long mg = ti.m_base + m;
  if (p.out_f32) {
    float* D = reinterpret_cast<float*>(p.D) + ti.d_off;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      if (n < ti.n_valid) {
        const long long ng = ti.n_base + n;
        if (p.trans_out) D[ng * p.ldd + mg] = v[j];
        else D[mg * p.ldd + ng] = v[j];
      }
    }
    return;
  }
  __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(p.D) + ti.d_off;
  if (p.trans_out) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      if (n < ti.n_valid) D[(long long)(ti.n_base + n) * p.ldd + mg] = __float2bfloat16_rn(v[j]);
    }
  } else {
    __nv_bfloat16* dst = D + mg * p.ldd + ti.n_base + c0;
    if (c0 + 16 <= ti.n_valid && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
      st_bf16x8(dst, v);
      st_bf16x8(dst + 8, v + 8);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < ti.n_valid) dst[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Tensor-parallel reduce-scatter epilogue: 16 fp32 partials of row m (tile
// columns c0..c0+15 = tokens) go to their owner ranks as tagged words. Lanes hold
// consecutive m, so a warp's stores to one token are 256 contiguous bytes.
template <int BN>
SP_DEVI void rs_store16(const GemmKParams& p, const TileInfo& ti, int m, int c0, const float (&v)[16], int ks,
                        uint32_t tag, int buf) {
  if (m >= ti.m_valid) return;
  const long long mg = ti.m_base + m;
  const int slots = p.tp_world * p.splits;
  const int slot = p.tp_rank * p.splits + ks;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int n = c0 + j;
    if (n < ti.n_valid) {
      const int ng = ti.n_base + n;
      const int owner = ng / p.tp_rows, nl = ng - owner * p.tp_rows;
      u64* dst = reinterpret_cast<u64*>(p.tp_base[owner] + p.tp_rs_off) +
                 ((((long long)buf * slots + slot) * p.tp_rows + nl) * p.M + mg);
      st_ll(dst, ll_word(__float_as_uint(v[j]), tag));
    }
  }
}

SP_DEVI uint32_t tp_tag(const GemmKParams& p, int* buf) {
  const u64 e = u64(*p.tp_epoch) * p.tp_layers_per_step + p.tp_layer;
  *buf = int(e & 1);
  return uint32_t(e + 1);
}

// All-gather operand: the producer warp waits until rows [0, n) of this layer's
// all-gather half are published (their flags carry `tag`); the 32 lanes poll
// disjoint rows at once, so the wait costs about one flag round trip. Then the
// async proxy (TMA) is ordered after the acquires. Bounded; false on a timeout
// (the same on every lane).
SP_DEVI bool ag_wait_rows_warp(const GemmKParams& p, int n, uint32_t tag, int buf) {
  const int lane = threadIdx.x & 31;
  const u64* f = p.tp_ag_flags + (long long)buf * p.tp_world * p.tp_rows;
  bool ok = true;
  for (int r = lane; r < n && ok; r += 32) {
    const long long t0 = clock64();
    for (unsigned it = 0;; ++it) {
      u64 v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f + r) : "memory");
      if (uint32_t(v) == tag) break;
      if (clock64() - t0 > p.tp_budget) { atomicCAS(p.err, 0, kErrWaitTimeoutPeer); ok = false; break; }
      if ((it & 255) == 255 && poll_abort(p.err)) { ok = false; break; }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return __all_sync(0xffffffffu, ok);
}

template <int BN, int MODE>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmKParams p) {
  using C = GemmCfg<BN, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_ntiles = s_err + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  float* xbuf = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    *s_err = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc<C::TMEM_COLS>(tmem_slot);
    tmem_relinquish();
    tc_fence_before();
  }
  // PDL: weights (A) never change while serving, so the producer may stream the
  // first stages of A before the previous kernel has finished; everything else
  // (B activations, outputs, device-side tile counts) waits for it.
  // (the all-gather operand's warp-wide flag wait needs the whole producer warp past the PDL wait)
  // Grouped: the tile count lives in device memory; with sched_early its writer is known
  // to have finished, so the weight-major grouped producer prefetches too.
  const bool sched_ready = MODE == MODE_GROUPED && p.sched_early && !p.ep_on;
  const bool prefetch_a = ((MODE != MODE_GROUPED && MODE != MODE_GROUPED_TM) || sched_ready) && p.a_evict_first &&
                          !p.tp_ag_flags;
  const bool is_producer = (warp == 0 && lane == 0);
  if ((MODE == MODE_GROUPED || MODE == MODE_GROUPED_TM) && !sched_ready) griddep_wait();
  if (threadIdx.x == 0) {
    int nt = p.num_tiles;
    if (MODE == MODE_GROUPED) nt = p.m_tiles * __ldg(p.grp_tiles + p.num_groups);
    if (MODE == MODE_GROUPED_TM) nt = p.n_tiles * __ldg(p.grp_tiles + p.num_groups);
    *s_ntiles = nt;
  }
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  if (!(prefetch_a && is_producer)) griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = *s_ntiles;


  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int ag_buf = 0;
    const uint32_t ag_tag = p.tp_ag_flags ? tp_tag(p, &ag_buf) : 0u;
    const bool ag_ok = !p.tp_ag_flags || ag_wait_rows_warp(p, p.N, ag_tag, ag_buf);
    if (!ag_ok && lane == 0) *s_err = kErrWaitTimeoutPeer;
    if (lane == 0 && ag_ok) {
      const uint64_t pol_a = p.a_evict_first ? policy_evict_first() : policy_evict_last();
      int it = 0;
      bool ok = true;
      int pre = 0;  // stages whose A tile went out before the PDL wait
      if (prefetch_a) {
        // A stages of the first work items, in the main loop's order
        WorkItem w0;
        for (int wi = 0; pre < C::STAGES && work_item<MODE>(p, num_tiles, wi, w0); ++wi) {
          TileInfo t0;
          get_tile<BN, MODE>(p, w0.tile, t0);
          for (int kb = w0.kb0; kb < w0.kb1 && pre < C::STAGES; ++kb, ++pre) {
            mbar_arrive_expect_tx(&full[pre], C::STAGE_BYTES);
            tma_load_2d_hint(smem + pre * C::STAGE_BYTES, &tmA, &full[pre], t0.a_k + kb * BK, t0.a_row, pol_a);
          }
        }
        griddep_wait();
      }
      // all-gather operand: rows of this layer's parity half (published, waited for above)
      const int ag_row0 = ag_buf * p.tp_world * p.tp_rows;
      WorkItem w;
      for (int wi = 0; ok && work_item<MODE>(p, num_tiles, wi, w); ++wi) {
        TileInfo ti;
        if (!get_tile<BN, MODE>(p, w.tile, ti)) continue;
        const int b_row = ti.b_row + ag_row0;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          if (it < pre) {
            tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], ti.b_k + kb * BK, b_row);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1, s_err, p.err, kErrWaitTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d_hint(sa, &tmA, &full[s], ti.a_k + kb * BK, ti.a_row, pol_a);
          tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], ti.b_k + kb * BK, b_row);
        }
      }
      if (!ok) {
        // Let loads already in flight land before the CTA releases its memory.
        for (int j = 0; j < C::STAGES && j < it; ++j) {
          const int i2 = it - 1 - j;
          mbar_wait(&full[i2 % C::STAGES], (i2 / C::STAGES) & 1, s_err, nullptr, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int it = 0, tc = 0;
      bool ok = true;
      WorkItem w;
      for (int wi = 0; ok && work_item<MODE>(p, num_tiles, wi, w); ++wi) {
        TileInfo ti;
        if (!get_tile<BN, MODE>(p, w.tile, ti)) continue;
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1, s_err, p.err, kErrWaitTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, s_err, p.err, kErrWaitTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t adesc = sdesc_kmajor_sw128(sa);
          const uint64_t bdesc = sdesc_kmajor_sw128(sa + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes of K per step -> +2 in the encoded start address
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > w.kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
        ++tc;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int m = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    if (MODE != MODE_SPLITK) {
      int tc = 0;
      WorkItem w;
      for (int wi = 0; work_item<MODE>(p, num_tiles, wi, w); ++wi) {
        TileInfo ti;
        if (!get_tile<BN, MODE>(p, w.tile, ti)) continue;
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait(&tfull[buf], tph, s_err, p.err, kErrWaitTimeoutEpilogue)) break;
        tc_fence_after();
        if (MODE == MODE_GROUPED_TM && p.swiglu) {
          // this thread's token row: columns [128 h, 128 h + 64) gate, the next 64 up.
          // tcgen05.ld is warp-collective, so every lane loads; only valid rows store.
          __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(p.D) +
                                (long long)(ti.m_base + min(m, ti.m_valid - 1)) * p.ldd + ti.n_base;
          for (int half = 0; half < BN / 128; ++half) {
            if (half * 128 >= ti.n_valid) break;
#pragma unroll 1
            for (int c0 = 0; c0 < 64; c0 += 16) {
              float g[16], u[16];
              tmem_ld16(lane_addr + buf * BN + half * 128 + c0, g);
              tmem_ld16(lane_addr + buf * BN + half * 128 + 64 + c0, u);
#pragma unroll
              for (int j = 0; j < 16; ++j) g[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
              if (m < ti.m_valid) {
                st_bf16x8(drow + half * 64 + c0, g);
                st_bf16x8(drow + half * 64 + c0 + 8, g + 8);
              }
            }
          }
        } else if (MODE == MODE_GROUPED && p.swiglu) {
          // rows [0, 64) of the tile are gate features, rows [64, 128) the matching
          // up features: exchange through shared memory, write silu(g) * u.
          __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(p.D);
          const int f = (ti.m_base >> 1) + m;
          for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + buf * BN + c0, v);
            if (m >= 64) {
#pragma unroll
              for (int j = 0; j < 16; ++j) xbuf[(m - 64) * 17 + j] = v[j];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (m < 64 && 2 * m < ti.m_valid) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (c0 + j < ti.n_valid) {
                  const float g = v[j], u = xbuf[m * 17 + j];
                  D[(long long)(ti.n_base + c0 + j) * p.ldd + f] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
                }
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        } else if (MODE == MODE_GROUPED && p.ep_on) {
          int ebuf;
          const uint32_t etag = ep_comb_tag(p.ep, &ebuf);
          for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + buf * BN + c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c0 + j < ti.n_valid)
                ep_comb_store(p.ep, ebuf, etag, ti.n_base + c0 + j, ti.m_base + m, v[j], m < ti.m_valid);
          }
        } else if (p.tp_rs) {
          int rbuf;
          const uint32_t tag = tp_tag(p, &rbuf);
          for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + buf * BN + c0, v);
            rs_store16<BN>(p, ti, m, c0, v, 0, tag, rbuf);
          }
        } else {
          for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + buf * BN + c0, v);
            store_chunk<BN>(p, ti, m, c0, v);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        ++tc;
      }
    } else {
      // Split-K: each work item's fp32 partial goes to slab `slot` of the workspace,
      // in the output's (n, m) coordinates with a dense pitch; the CTA that finishes a
      // tile (its last slot) zeroes the tile's slots the stream-K split leaves unused.
      int tc = 0;
      WorkItem w;
      for (int wi = 0; work_item<MODE>(p, num_tiles, wi, w); ++wi) {
        TileInfo ti;
        get_tile<BN, MODE>(p, w.tile, ti);
        GemmKParams q = p;
        q.out_f32 = 1;
        q.ldd = p.trans_out ? p.M : p.N;
        ti.d_off = 0;
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait(&tfull[buf], tph, s_err, p.err, kErrWaitTimeoutEpilogue)) break;
        tc_fence_after();
        int rbuf = 0;
        const uint32_t tag = p.tp_rs ? tp_tag(p, &rbuf) : 0u;
        q.D = p.ws + (size_t)w.slot * p.split_stride;
        for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) {
          float v[16];
          tmem_ld16(lane_addr + buf * BN + c0, v);
          if (p.tp_rs) rs_store16<BN>(p, ti, m, c0, v, w.slot, tag, rbuf);
          else store_chunk<BN>(q, ti, m, c0, v);
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        ++tc;
        if (p.sk_ctas > 0 && w.slot == w.nseg - 1) {
          const float z[16] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int sl = w.nseg; sl < p.sk_slots; ++sl) {
            q.D = p.ws + (size_t)sl * p.split_stride;
            for (int c0 = 0; c0 < BN && c0 < ti.n_valid; c0 += 16) store_chunk<BN>(q, ti, m, c0, z);
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<C::TMEM_COLS>(tmem_base);
  }
}

// Sums the split-K slabs: out[r, c] = sum_s ws[s][r][c] for a [rows, cols]
// dense slab layout; output pitch ldo (elements), bf16 or fp32.
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ ws, long long stride,
                                                           int splits, int rows, int cols, void* __restrict__ out,
                                                           long long ldo, int out_f32) {
  griddep_wait();
  griddep_launch();
  const int c4 = cols / 4;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * c4) return;
  const int r = int(i / c4), c = int(i % c4) * 4;
  const float* src = ws + (long long)r * cols + c;
  float4 acc = __ldcg(reinterpret_cast<const float4*>(src));
  for (int s = 1; s < splits; ++s) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + s * stride));
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (out_f32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (long long)r * ldo + c) = acc;
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + (long long)r * ldo + c;
    *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(acc.x, acc.y);
    *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(acc.z, acc.w);
  }
}

// ======================================================================= host

void split_reduce(const float* ws, long long stride, int splits, int rows, int cols, void* out, long long ldo,
                  int out_f32, cudaStream_t s) {
  const long long n = (long long)rows * (cols / 4);
  launch_k(split_reduce_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, ws, stride, splits, rows, cols,
           out, ldo, out_f32);
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
      throw std::runtime_error("sparkpipe: cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<PFN_encodeTiled>(ptr);
  }
  return fn;
}

// 2-D K-major tensor map: `rows` x `cols` elements, row pitch `ld` elements, box
// (box_cols x box_rows), 128-byte swizzle, zero fill outside the tensor.
void make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, long long rows,
                  long long cols, long long ld, int box_rows, int box_cols) {
  make_tmap_2d_swizzle(map, ptr, dt, elem_bytes, rows, cols, ld, box_rows, box_cols, CU_TENSOR_MAP_SWIZZLE_128B);
}

void make_tmap_2d_swizzle(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, long long rows,
                          long long cols, long long ld, int box_rows, int box_cols, CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) throw std::runtime_error("tensor map base not 16B aligned");
  if ((ld * elem_bytes) % 16 != 0) throw std::runtime_error("tensor map row pitch not a multiple of 16 bytes");
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = get_encode_fn()(map, dt, 2, const_cast<void*>(ptr), gdim, gstride, box, estride,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

template <int BN, int MODE>
static void launch_gemm(const GemmLaunch& g, GemmKParams& p) {
  using C = GemmCfg<BN, MODE>;
  CUtensorMap ta, tb;
  make_tmap_2d(&ta, g.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.a_rows, g.a_cols, g.lda, BM, BK);
  make_tmap_2d(&tb, g.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.b_rows, g.b_cols, g.ldb, BN, BK);
  auto kern = gemm_bf16_kernel<BN, MODE>;
  set_smem_bytes(kern, C::SMEM_BYTES);
  prefer_max_smem_carveout(reinterpret_cast<const void*>(kern));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attrs[2];
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = g.stream;
  if (MODE == MODE_SPLITK) {
    cfg.gridDim = dim3(p.sk_ctas > 0 ? p.sk_ctas : p.num_tiles * p.splits, 1, 1);
    cfg.attrs = attrs;
    cfg.numAttrs = 0;
  } else {
    int grid = (MODE == MODE_GROUPED || MODE == MODE_GROUPED_TM) ? g.num_sms : std::min(p.num_tiles, g.num_sms);
    if (grid < 1) grid = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.attrs = attrs;
    cfg.numAttrs = 0;
  }
  if (pdl_enabled()) {
    attrs[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs += 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm launch failed: ") + cudaGetErrorString(e));
}

template <int MODE>
static void dispatch_bn(int bn, const GemmLaunch& g, GemmKParams& p) {
  switch (bn) {
    case 16: launch_gemm<16, MODE>(g, p); break;
    case 32: launch_gemm<32, MODE>(g, p); break;
    case 64: launch_gemm<64, MODE>(g, p); break;
    case 128: launch_gemm<128, MODE>(g, p); break;
    case 256: launch_gemm<256, MODE>(g, p); break;
    default: throw std::runtime_error("unsupported BLOCK_N");
  }
}

static int pick_bn(int n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

static int pick_or(const GemmLaunch& g, const GemmKParams&) { return g.block_n > 0 ? g.block_n : pick_bn(g.N); }

static void check_k_window(long long cols, int k0, int batch_k, int K, int batch) {
  const long long kmax = (long long)k0 + (long long)batch_k * (batch - 1) + K;
  if (kmax > cols) throw std::runtime_error("gemm: K window exceeds operand columns");
  const bool partial = (k0 != 0) || (batch_k != 0) || (K != cols);
  if (partial && (K % BK) != 0)
    throw std::runtime_error("gemm: a K window inside a wider operand needs K % 64 == 0");
}

int gemm_bf16(const GemmLaunch& g) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return 0;
  if (g.K % 8 != 0) throw std::runtime_error("gemm: K must be a multiple of 8");
  check_k_window(g.a_cols, g.a_k0, g.a_batch_k, g.K, g.grouped ? 1 : g.batch);
  check_k_window(g.b_cols, g.b_k0, g.b_batch_k, g.K, g.grouped ? 1 : g.batch);
  GemmKParams p = {};
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.batch = g.batch;
  p.a_row0 = g.a_row0; p.a_batch_rows = g.a_batch_rows; p.a_k0 = g.a_k0; p.a_batch_k = g.a_batch_k;
  p.b_row0 = g.b_row0; p.b_batch_rows = g.b_batch_rows; p.b_k0 = g.b_k0; p.b_batch_k = g.b_batch_k;
  p.D = g.D; p.ldd = g.ldd; p.d_batch_stride = g.d_batch_stride;
  p.trans_out = g.trans_out; p.out_f32 = g.out_f32;
  p.err = g.err;
  p.a_evict_first = g.a_evict_first;
  p.sched_early = g.sched_early;
  p.swiglu = g.swiglu;
  if (g.swiglu && g.grouped != 2 && (!g.grouped || !g.trans_out || g.out_f32 || g.M % 128 != 0))
    throw std::runtime_error("gemm: fused SwiGLU needs a grouped, transposed bf16 GEMM with M % 128 == 0");
  p.m_tiles = (g.M + BM - 1) / BM;
  if (g.tp) {
    const TpGemm& t = *g.tp;
    if (g.grouped || g.batch != 1) throw std::runtime_error("gemm: tensor-parallel operands need a plain GEMM");
    if (!t.epoch || t.world < 1 || t.world > 8 || t.rank < 0 || t.rank >= t.world || t.rows <= 0)
      throw std::runtime_error("gemm: bad tensor-parallel arguments");
    for (int r = 0; r < t.world; ++r)
      if (!t.base[r] || (t.base[r] & 255)) throw std::runtime_error("gemm: bad tensor-parallel rank base");
    if (t.rs && (!g.trans_out || g.N > t.world * t.rows))
      throw std::runtime_error("gemm: reduce-scatter needs a transposed output over world x rows tokens");
    if (t.ag_flags && (g.N > t.world * t.rows || g.b_rows != 2ll * t.world * t.rows))
      throw std::runtime_error("gemm: the all-gather operand is the [2 x world x rows, K] region");
    for (int r = 0; r < 8; ++r) p.tp_base[r] = t.base[r];
    p.tp_rs_off = t.rs_off; p.tp_rs = t.rs; p.tp_rank = t.rank; p.tp_world = t.world; p.tp_rows = t.rows;
    p.tp_ag_flags = static_cast<const unsigned long long*>(t.ag_flags);
    p.tp_epoch = t.epoch; p.tp_layer = t.layer; p.tp_layers_per_step = t.layers_per_step; p.tp_budget = t.budget;
  }
  if (g.ep) {
    if (!g.grouped || !g.trans_out || g.out_f32 || g.swiglu || g.M != g.ep->H || g.ep->H % 2)
      throw std::runtime_error("gemm: the combine epilogue needs a grouped, transposed bf16 GEMM with M = hidden");
    p.ep_on = 1;
    const EpComb& e = *g.ep;
    for (int r = 0; r < 8; ++r) p.ep.base[r] = e.base[r];
    p.ep.comb_off = e.comb_off; p.ep.cap = e.cap; p.ep.kk = e.kk; p.ep.H = e.H;
    p.ep.layers_per_step = e.layers_per_step; p.ep.comb_dst = e.comb_dst; p.ep.epoch = e.epoch; p.ep.layer = e.layer;
  }
  if (g.grouped == 2) {  // token-major: tokens as A (M), weights as B (N), row-major output
    const int bn = g.block_n > 0 ? g.block_n : 256;
    if (g.trans_out || g.out_f32 || g.tp || g.ep || (bn != 128 && bn != 256))
      throw std::runtime_error("gemm: the token-major grouped GEMM writes bf16 rows with BLOCK_N 128 or 256");
    if (g.swiglu && (g.N % bn != 0 || g.ldd % 8 != 0 || (reinterpret_cast<uintptr_t>(g.D) & 15)))
      throw std::runtime_error("gemm: token-major SwiGLU needs N % BLOCK_N == 0 and 16-byte output rows");
    p.n_tiles = (g.N + bn - 1) / bn;
    p.num_tiles = 0;
    p.grp_rows = g.grp_rows;
    p.grp_tiles = g.grp_tiles;
    p.num_groups = g.num_groups;
    if (bn == 256) launch_gemm<256, MODE_GROUPED_TM>(g, p);
    else launch_gemm<128, MODE_GROUPED_TM>(g, p);
    return 1;
  }
  if (g.grouped) {
    const int bn = g.block_n > 0 ? g.block_n : 32;
    p.n_tiles = 0;
    p.num_tiles = 0;
    p.grp_rows = g.grp_rows;
    p.grp_tiles = g.grp_tiles;
    p.num_groups = g.num_groups;
    dispatch_bn<MODE_GROUPED>(bn, g, p);
    return 1;
  }
  const int bn = pick_or(g, p);
  p.n_tiles = (g.N + bn - 1) / bn;
  p.num_tiles = p.m_tiles * p.n_tiles * g.batch;
  int splits = g.splits;
  const int kbs = (g.K + BK - 1) / BK;
  const long long slab = (long long)g.M * g.N;
  const int out_cols = g.trans_out ? g.M : g.N;
  // partial slabs need dense, 4-aligned rows, a workspace, and (reduced here) an aligned output
  const bool slabs_ok = g.ws && g.batch == 1 && out_cols % 4 == 0 &&
                        (g.slab_out || (g.ldd % 4 == 0 && (reinterpret_cast<uintptr_t>(g.D) & 15) == 0));
  // The fixed split below keeps one CTA per SM: tiles x splits <= SMs.
  const int fixed_splits = std::max(1, std::min({g.num_sms / std::max(1, p.num_tiles), kbs / 2, 16}));
  static const bool streamk_on = [] {
    const char* e = std::getenv("SPARKPIPE_GEMM_STREAMK");
    return !(e && e[0] == '0');
  }();
  // Between half the SMs and all of them in tiles, a fixed split of two keeps every CTA
  // resident at once (two per SM fit beside each other) with two partial slabs per tile:
  // 64 x 9792 x 2048 measured 13.8 us against 16.1 us for the stream-K split (which
  // leaves up to three slabs per tile and CTAs that finish two tiles).
  const int splitk_smem = GemmCfg<16, MODE_SPLITK>::STAGES * (BM + bn) * BK * 2 + 1024 + 256 + 64 * 17 * 4;
  const bool two_way = splits <= 0 && !g.tp && slabs_ok && kbs >= 4 && 2 * p.num_tiles > g.num_sms &&
                       p.num_tiles <= g.num_sms && 2 * splitk_smem <= 227 * 1024;
  if (two_way) splits = 2;
  if (streamk_on && splits <= 0 && !g.tp && slabs_ok && p.num_tiles >= 8 &&
      p.num_tiles * fixed_splits * 10 < g.num_sms * 6 && kbs >= 2) {
    // Stream-K split, when the fixed split would leave over 40% of the SMs idle and
    // there are enough tiles to share (77 tiles on 148 SMs: one split, 77 CTAs): the (tile, K-block) units are spread
    // evenly over one CTA per SM, a tile's K range shared by consecutive CTAs. G is
    // lowered until no tile needs more than 16 partial slots. Measured (64 tokens,
    // K 2048, 9792 rows): 16.4 -> 15.9 us; where the fixed split fills the SMs it is
    // faster (2048 rows: 9.2 us fixed vs 11.3 us stream-K).
    const long long T = (long long)p.num_tiles * kbs;
    auto cta_of = [](long long w, long long W, int G) { return int(((w + 1) * G + W - 1) / W) - 1; };
    int G = (int)std::min<long long>(g.num_sms, T), slots = 0;
    for (; G >= 1; --G) {
      slots = 0;
      for (int t = 0; t < p.num_tiles; ++t)
        slots = std::max(slots, cta_of((long long)t * kbs + kbs - 1, T, G) - cta_of((long long)t * kbs, T, G) + 1);
      if (slots <= 16) break;
    }
    if (G > p.num_tiles && slots > 1 && slab * slots <= g.ws_floats) {
      p.ws = g.ws;
      p.split_stride = slab;
      p.splits = slots;
      p.sk_ctas = G;
      p.sk_slots = slots;
      dispatch_bn<MODE_SPLITK>(pick_or(g, p), g, p);
      if (g.slab_out) return -slots;
      const int rows = g.trans_out ? g.N : g.M;
      split_reduce(g.ws, slab, slots, rows, out_cols, g.D, g.ldd, g.out_f32, g.stream);
      return 2;
    }
  }
  if (splits <= 0) {
    // Auto: the most splits that keep one CTA per SM (tiles x splits <= SMs), at
    // least two K blocks per split, at most 16. Each SM streams its own share of
    // the weights: two CTAs on some SMs and one on others leaves the doubled SMs as
    // the tail. (64 x 3648 x 2048: 5 splits, 145 CTAs; the old power-of-two rule
    // chose 8 splits, 232 CTAs.)
    splits = fixed_splits;
  }
  if (splits > kbs) splits = kbs;  // every split CTA needs at least one K block
  if (g.tp && g.tp->rs) {
    // partials go straight to the owners' slots: no workspace, no reduction kernel
    splits = std::max(1, std::min(splits, g.tp->max_splits));
    p.splits = splits;
    if (splits > 1) dispatch_bn<MODE_SPLITK>(bn, g, p);
    else dispatch_bn<MODE_DENSE>(bn, g, p);
    return 1;
  }
  // the slab reduction needs dense, 4-aligned rows and a workspace that fits
  if (splits > 1 && (!slabs_ok || slab * splits > g.ws_floats)) splits = 1;
  p.ws = g.ws;
  p.split_stride = slab;
  p.splits = splits;
  if (splits > 1) {
    dispatch_bn<MODE_SPLITK>(bn, g, p);
    if (g.slab_out) return -splits;  // the caller's next kernel sums the slabs itself
    const int rows = g.trans_out ? g.N : g.M;
    const int cols = g.trans_out ? g.M : g.N;
    split_reduce(g.ws, slab, splits, rows, cols, g.D, g.ldd, g.out_f32, g.stream);
    return 2;
  }
  dispatch_bn<MODE_DENSE>(bn, g, p);
  return 1;
}

void kernel_attrs_gemm(std::vector<KernelAttr>& out) {
#define SP_GEMM_ATTR(BN, MODE) push_kernel_attr(out, "gemm_bf16_kernel<" #BN "," #MODE ">", gemm_bf16_kernel<BN, MODE>)
  SP_GEMM_ATTR(16, 0); SP_GEMM_ATTR(32, 0); SP_GEMM_ATTR(64, 0); SP_GEMM_ATTR(128, 0); SP_GEMM_ATTR(256, 0);
  SP_GEMM_ATTR(16, 1); SP_GEMM_ATTR(32, 1); SP_GEMM_ATTR(64, 1); SP_GEMM_ATTR(128, 1); SP_GEMM_ATTR(256, 1);
  SP_GEMM_ATTR(16, 2); SP_GEMM_ATTR(32, 2); SP_GEMM_ATTR(64, 2); SP_GEMM_ATTR(128, 2); SP_GEMM_ATTR(256, 2);
#undef SP_GEMM_ATTR
}

}  // namespace sp
