// MLA paged latent-KV decode attention with a flattened (stream-K) schedule, sm_100a.
//
// Same computation as mla_decode.cu (absorbed form: for sequence b, head h,
// o[b,h,:] = softmax(scale * q[b,h,:] . K^T) V over the sequence's paged cache
// rows [latent 512 | rope 64], V = the latent part), organised for a decode batch
// whose KV stream has to fill the whole GPU:
//
// * Schedule. The work is cut into 32-token units (half a 64-token cache block).
//   Row r = (sequence b, head group g), in the order b-major so that the head groups
//   of one sequence are adjacent (their shared KV is read by neighbouring CTAs at
//   about the same time, the second read from L2), owns ceil(ctx_b / 32) units. The
//   rows' units are laid end to end and CTA c of G takes units [c*W/G, (c+1)*W/G),
//   so every SM streams the same number of KV bytes whatever the mix of context
//   lengths, with no partial second wave. Each CTA computes the prefix sums of the
//   units itself from context_lens (one block-wide scan): no host work, no extra
//   kernel, and the launch is CUDA-graph safe.
// * Pieces. A CTA's range crosses row boundaries; each (row, unit range) piece is
//   one online-softmax pass. A piece that covers its whole row writes the bf16
//   output directly; otherwise it writes a normalised fp32 partial and its
//   log-sum-exp to segment c + r (unique: c + r grows strictly along the unit
//   order), bumps the row's arrival counter, and the CTA that arrives last merges
//   the row's segments and resets the counter for the next launch. No CTA ever
//   waits on another.
// * Pipeline. One producer warp streams 36 KB stages (32 tokens x 576 bf16, nine
//   128-byte-swizzled TMA boxes) through a ring. Four consumer warps per 16-head
//   tile run mma.sync (m16n8k16, bf16 -> fp32): warp j computes the partial scores
//   of all 32 tokens over its quarter of the 576 dims (k-steps [9j, 9j+9), four
//   independent accumulator chains, so each query byte is read from shared memory
//   once per stage rather than once per warp); the partials meet in a
//   double-buffered shared slab behind one barrier, after which every warp holds the
//   full 16 x 32 scores in accumulator layout, runs the online softmax itself and
//   feeds P straight from registers as the A operand of O += P V for its 128 latent
//   dims. One barrier per stage, no P or row-max exchange through shared memory.
// * Occupancy. The 16-head kernel fits two CTAs per SM (two stages each), so each
//   SM sub-partition interleaves two consumer warps.
// * PDL. In a CUDA graph (`early`), only the cache row of the newest token is
//   written by the kernel before this one (the prep kernel); rows of earlier
//   positions and the schedule inputs were written by earlier graph launches or
//   copied in before the launch. The producer therefore issues the first stages
//   that do not hold a sequence's newest token before the grid-dependency wait, so
//   the first bytes are in flight while the prep kernel finishes. Outside a graph
//   the kernel waits first.
//
// Reference: PHASE_MLA_ATTENTION with ABSORBED_LATENT mode and block tables in
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:445-460,
// 563-568; the scheduling here is this framework's own.
#include <cuda_runtime.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "mma_sync.cuh"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace mlask {

constexpr int TOK = 32;    // tokens per unit / stage
constexpr int DIM = 576;   // kv_lora 512 + rope 64
constexpr int LAT = 512;
constexpr int CH = 9;      // 64-column (128-byte) chunks of a row
constexpr int BLK = 64;    // tokens per cache block
constexpr int NJ = 4;      // consumer warps per 16-head tile
constexpr int KS = DIM / 16 / NJ;  // k-steps of S per warp (9)
constexpr int MAX_B = 1024;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

template <int HT, int MINB>
struct Cfg {
  static constexpr int HG = 16 * HT;                 // heads per CTA
  static constexpr int CW = NJ * HT;                 // consumer warps
  static constexpr int CT = CW * 32;                 // consumer threads
  static constexpr int THREADS = CT + 32;            // + producer warp
  static constexpr int STAGES = MINB == 2 ? 2 : (HT == 1 ? 5 : 3);
  static constexpr int STAGE_BYTES = CH * TOK * 128;
  static constexpr int Q_BYTES = CH * HG * 128;
  static constexpr int DIMW = LAT / NJ;              // latent dims per warp in O
  static constexpr int NP = DIMW / 16;               // n8-tile pairs per warp in O
  static constexpr int PART_BYTES = 2 * HT * NJ * 4 * 32 * 16;  // [2][HT][NJ][4 tiles][32 lanes] float4
  static constexpr int OFF_KV = align_up(Q_BYTES, 1024);
  static constexpr int OFF_PART = OFF_KV + STAGES * STAGE_BYTES;
  static constexpr int OFF_STAT = OFF_PART + PART_BYTES;
  static constexpr int OFF_SCAN = OFF_STAT + 2 * HG * 4;
  static constexpr int OFF_BAR = align_up(OFF_SCAN + (MAX_B + 1 + 16) * 4, 8);
  static constexpr int NBAR = 2 * STAGES + 2;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + alignment slack
  static_assert(MINB * (SMEM + 1024) <= 228 * 1024, "shared memory per SM");
  static_assert(THREADS / 32 <= 16, "scan scratch");
};

struct Params {
  const int* block_table;
  int max_blocks;
  const int* context_lens;
  bf16* out;           // [B, H, 512]
  float* o_part;       // [segments][HG][512]
  float* lse_part;     // [segments][HG]
  int* counters;       // [B * NG], zero between launches
  int B, H, NG;
  float scale_log2;
  int early;
  int* err;
  unsigned long long* trace;  // optional: [4 CTAs][64] global-timer stamps (diagnostics)
};

// Trace slots of one CTA: 0 start, 1 schedule ready, 2 producer past the dependency
// wait, 3 + 2i / 4 + 2i: piece i queries landed / piece i finished (i < 8),
// 60 merge start, 61 merge end, 63 consumers done. (Nothing inside the stage loop: a
// timer read there costs throughput.)
SP_DEVI void sk_mark(const Params& p, int slot) {
  if (p.trace == nullptr) return;
  const int G = gridDim.x;
  const int which = blockIdx.x == 0 ? 0 : blockIdx.x == 1 ? 1 : blockIdx.x == G / 2 ? 2 : blockIdx.x == G - 1 ? 3 : -1;
  if (which >= 0 && slot < 64) p.trace[which * 64 + slot] = globaltimer();
}

SP_DEVI void cbar(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }
SP_DEVI bool cbar_and(bool v, int n) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(n)
      : "memory");
  return r != 0;
}

// CTA owning flattened unit w when W units are split over G CTAs.
SP_DEVI int cta_of(long long w, long long W, int G) { return int(((w + 1) * G + W - 1) / W) - 1; }

// Units of sequence b.
SP_DEVI int units_of(const Params& p, int b) {
  const int ctx = min(max(p.context_lens[b], 0), p.max_blocks * BLK);
  return (ctx + TOK - 1) / TOK;
}

// A piece of this CTA's range: row r = b * NG + g, units [u0, u1) of the row's n
// units, and the row's first unit in the flattened order.
struct Piece {
  int g, b, r, u0, u1, n;
  long long row_w0;
};

// Row holding flattened unit w: the rows of sequence b occupy [NG*sW[b], NG*sW[b+1]).
SP_DEVI Piece piece_at(const int* sW, int B, int NG, long long w, long long w_end) {
  Piece pc;
  const int wq = int(w / NG);
  int lo = 0, hi = B;  // last b with sW[b] <= wq (skips empty sequences)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sW[mid] <= wq) lo = mid; else hi = mid;
  }
  pc.b = lo;
  pc.n = sW[lo + 1] - sW[lo];
  const long long off = w - (long long)NG * sW[lo];
  pc.g = int(off / pc.n);
  pc.r = lo * NG + pc.g;
  pc.u0 = int(off - (long long)pc.g * pc.n);
  pc.u1 = int(min((long long)pc.n, pc.u0 + (w_end - w)));
  pc.row_w0 = (long long)NG * sW[lo] + (long long)pc.g * pc.n;
  return pc;
}

template <int HT, int MINB>
__global__ void __launch_bounds__(Cfg<HT, MINB>::THREADS, MINB)
    mla_decode_sk_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const Params p) {
  using C = Cfg<HT, MINB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  float4* sPart = reinterpret_cast<float4*>(smem + C::OFF_PART);
  float* sM = reinterpret_cast<float*>(smem + C::OFF_STAT);  // [HG] combine: row max
  float* sS = sM + C::HG;                                      // [HG] combine: 1 / normaliser
  int* sW = reinterpret_cast<int*>(smem + C::OFF_SCAN);        // [B + 1] unit prefix sums
  int* sWarp = sW + MAX_B + 1;                                  // [16] scan scratch
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + C::STAGES;
  uint64_t* qfull = empty + C::STAGES;
  uint64_t* qempty = qfull + 1;
  volatile int* s_err = reinterpret_cast<volatile int*>(qempty + 1);
  volatile int* s_flag = s_err + 1;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int B = p.B, NG = p.NG;

  if (tid == 0) {
    sk_mark(p, 0);
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], C::CW);
    }
    mbar_init(qfull, 1);
    mbar_init(qempty, C::CW);
    *s_err = 0;
    fence_mbarrier_init();
  }
  if (!p.early) {
    griddep_wait();
    griddep_launch();
  }
  // ---- units per sequence, exclusive prefix sums in sW[0..B]
  {
    const int per = (B + C::THREADS - 1) / C::THREADS;
    const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
    int sum = 0;
    for (int b = b0; b < b1; ++b) sum += units_of(p, b);
    int inc = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) sWarp[warp] = inc;
    __syncthreads();
    if (tid == 0) {
      int run = 0;
      for (int i = 0; i < C::THREADS / 32; ++i) {
        const int v = sWarp[i];
        sWarp[i] = run;
        run += v;
      }
      sW[B] = run;
    }
    __syncthreads();
    int run = sWarp[warp] + inc - sum;
    for (int b = b0; b < b1; ++b) {
      sW[b] = run;
      run += units_of(p, b);
    }
    __syncthreads();
  }
  if (tid == 0) sk_mark(p, 1);
  const int U = sW[B];
  const long long W = (long long)NG * U;
  // units go to the first min(grid, W) CTAs, so every working CTA owns at least one
  // unit and a row's segments come from consecutive CTAs c_first..c_last
  const int c = blockIdx.x;
  const int G = (W > 0 && W < gridDim.x) ? int(W) : int(gridDim.x);
  const long long w_begin = c < G ? W * c / G : 0, w_end = c < G ? W * (c + 1) / G : 0;

  if (warp == C::CW) {
    // ================================================================ producer warp
    if (lane != 0) {
      if (p.early) {
        griddep_wait();
        griddep_launch();
      }
      return;
    }
    bool waited = !p.early;
    auto wait_dep = [&]() {
      if (!waited) {
        griddep_wait();
        griddep_launch();
        waited = true;
        sk_mark(p, 2);
      }
    };
    auto issue_q = [&](const Piece& pc) {
      mbar_arrive_expect_tx(qfull, C::Q_BYTES);
      const int row = pc.b * p.H + pc.g * C::HG;
#pragma unroll 1
      for (int ch = 0; ch < CH; ++ch) tma_load_2d(smem + ch * C::HG * 128, &tmQ, qfull, ch * 64, row);
    };
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmKV);
    int it = 0, pieces = 0, q_issued = 0;
    bool ok = true;
    for (long long w = w_begin; w < w_end && ok; ++pieces) {
      const Piece pc = piece_at(sW, B, NG, w, w_end);
      w += pc.u1 - pc.u0;
      const int* bt = p.block_table + (long long)pc.b * p.max_blocks;
      const int ctx = min(max(p.context_lens[pc.b], 0), p.max_blocks * BLK);
      // Queries of piece 0 need the dependency wait (deferred in early mode until a
      // stage needs it). A later piece reuses the query buffer once the consumers
      // are past the previous piece's last score product; its stages go out
      // meanwhile, but before the ring wraps into the piece (the consumers need its
      // queries to free that slot) the query issue is forced.
      bool q_done = false;
      auto try_q = [&](bool force) -> bool {
        if (q_done) return true;
        if (pieces == 0) {
          if (!waited) return true;
        } else if (force) {
          if (!mbar_wait(qempty, (pieces - 1) & 1, s_err, p.err, kErrWaitTimeoutProducer)) return false;
        } else if (!mbar_test_wait(qempty, (pieces - 1) & 1)) {
          return true;
        }
        issue_q(pc);
        ++q_issued;
        q_done = true;
        return true;
      };
      for (int u = pc.u0; u < pc.u1; ++u, ++it) {
        const bool newest = (u + 1) * TOK >= ctx;  // holds the row the prep kernel writes
        if (!waited && (newest || it >= C::STAGES)) wait_dep();
        if (!try_q(u - pc.u0 >= C::STAGES)) { ok = false; break; }
        const int s = it % C::STAGES;
        if (it >= C::STAGES &&
            !mbar_wait(&empty[s], ((it / C::STAGES) - 1) & 1, s_err, p.err, kErrWaitTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        const int row = __ldg(bt + u / 2) * BLK + (u & 1) * TOK;
        uint8_t* dst = smem + C::OFF_KV + s * C::STAGE_BYTES;
#pragma unroll 1
        for (int ch = 0; ch < CH; ++ch) tma_load_2d(dst + ch * TOK * 128, &tmKV, &full[s], ch * 64, row);
      }
      if (ok) {
        wait_dep();
        if (!try_q(true)) ok = false;
      }
    }
    wait_dep();
    if (!ok) {
      // let copies already in flight land before the CTA's shared memory is released
      for (int i = max(0, it - C::STAGES); i < it; ++i) mbar_drain(&full[i % C::STAGES], (i / C::STAGES) & 1);
      if (q_issued > 0) mbar_drain(qfull, (q_issued - 1) & 1);
    }
    return;
  }

  // ================================================================== consumer warps
  const int mt = warp / NJ, j = warp % NJ;  // head tile; k-slice of S and dim slice of O
  const int r_lo = lane >> 2;
  const int qrow = mt * 16;
  const uint32_t sKV = smem_u32(smem + C::OFF_KV);
  int it = 0, pieces = 0;
  bool ok = true;
  bool launched = !p.early;
  for (long long w = w_begin; w < w_end && ok; ++pieces) {
    const Piece pc = piece_at(sW, B, NG, w, w_end);
    w += pc.u1 - pc.u0;
    const int ctx = min(max(p.context_lens[pc.b], 0), p.max_blocks * BLK);
    ok = cbar_and(mbar_wait(qfull, pieces & 1, s_err, p.err, kErrWaitTimeoutMma), C::CT);
    if (!ok) break;
    if (tid == 0 && pieces < 8) sk_mark(p, 3 + 2 * pieces);
    if (!launched) {
      griddep_launch();  // queries landed: the kernel before this one has completed
      launched = true;
    }
    float o[2 * C::NP][4];
#pragma unroll
    for (int n = 0; n < 2 * C::NP; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};
    for (int u = pc.u0; u < pc.u1; ++u, ++it) {
      const int s = it % C::STAGES;
      const bool got = mbar_wait(&full[s], (it / C::STAGES) & 1, s_err, p.err, kErrWaitTimeoutMma);
      const uint32_t kvb = sKV + s * C::STAGE_BYTES;
      // ---- partial S over this warp's 144 dims: 16 heads x 32 tokens (4 n8 tiles)
      float sc[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.f;
      if (got) {
#pragma unroll 3
        for (int kk = 0; kk < KS; ++kk) {
          const int k2 = j * KS + kk;
          uint32_t a[4];
          ldsm_x4(a, swz128(sQ + (k2 >> 2) * C::HG * 128, qrow + (lane & 15), (k2 & 3) * 16 + (lane >> 4) * 8));
          const uint32_t chb = kvb + (k2 >> 2) * TOK * 128;
          const int cc = (k2 & 3) * 16 + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int tp = 0; tp < 2; ++tp) {
            uint32_t bb[4];
            ldsm_x4(bb, swz128(chb, tp * 16 + (lane & 7) + (lane >> 4) * 8, cc));
            mma16816(sc[2 * tp], a, bb[0], bb[1]);
            mma16816(sc[2 * tp + 1], a, bb[2], bb[3]);
          }
        }
      }
      if (u + 1 == pc.u1) {
        // last score product of the piece: the query buffer may take the next piece
        __syncwarp();
        if (lane == 0) mbar_arrive(qempty);
      }
      float4* part = sPart + ((size_t)((it & 1) * HT + mt) * NJ) * 128;  // [NJ][4 tiles][32 lanes]
#pragma unroll
      for (int t = 0; t < 4; ++t) part[(j * 4 + t) * 32 + lane] = make_float4(sc[t][0], sc[t][1], sc[t][2], sc[t][3]);
      if (!cbar_and(got, C::CT)) { ok = false; break; }
      // ---- full scores: sum of the four k-slices, scale, mask, row max
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float4 a = part[t * 32 + lane];
#pragma unroll
        for (int jj = 1; jj < NJ; ++jj) {
          const float4 v = part[(jj * 4 + t) * 32 + lane];
          a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
        }
        sc[t][0] = a.x; sc[t][1] = a.y; sc[t][2] = a.z; sc[t][3] = a.w;
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int tok = u * TOK + t * 8 + (lane & 3) * 2;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = sc[t][e] * p.scale_log2;
          if (tok + (e & 1) >= ctx) v = -INFINITY;
          sc[t][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float mn = fmaxf(m_run[h], mx[h]);
        alpha[h] = (m_run[h] == -INFINITY) ? 0.f : fast_exp2(m_run[h] - mn);
        m_run[h] = mn;
        l_run[h] *= alpha[h];
      }
      // ---- P = exp2(S - m) as the A operand of P V (two k-steps of 16 tokens)
      uint32_t pa[2][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          pv[e] = (sc[t][e] == -INFINITY) ? 0.f : fast_exp2(sc[t][e] - m_run[e >> 1]);
          l_run[e >> 1] += pv[e];
        }
        pa[t >> 1][(t & 1) * 2 + 0] = pack_bf16(pv[0], pv[1]);
        pa[t >> 1][(t & 1) * 2 + 1] = pack_bf16(pv[2], pv[3]);
      }
#pragma unroll
      for (int n = 0; n < 2 * C::NP; ++n) {
        o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
        o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
      }
      // ---- O[16 heads, DIMW dims of slice j] += P[16, 32] V[32, DIMW]
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int tok = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int np = 0; np < C::NP; ++np) {
          const int dim = j * C::DIMW + np * 16 + (lane >> 4) * 8;
          uint32_t bb[4];
          ldsm_x4_t(bb, swz128(kvb + (dim >> 6) * TOK * 128, tok, dim & 63));
          mma16816(o[2 * np], pa[ks], bb[0], bb[1]);
          mma16816(o[2 * np + 1], pa[ks], bb[2], bb[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) break;
    if (tid == 0 && pieces < 8) sk_mark(p, 4 + 2 * pieces);

    // ---- finish the piece (every warp holds the complete row statistics)
    float inv[2], lse[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float l = l_run[h];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      inv[h] = l > 0.f ? 1.f / l : 0.f;
      lse[h] = l > 0.f ? m_run[h] + __log2f(l) : -INFINITY;
    }
    const int head_l0 = qrow + r_lo;  // head within the group (and +8)
    if (pc.u0 == 0 && pc.u1 == pc.n) {
      // the whole row in this CTA: final output
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        bf16* orow = p.out + ((long long)pc.b * p.H + pc.g * C::HG + head_l0 + h * 8) * LAT + j * C::DIMW +
                     (lane & 3) * 2;
#pragma unroll
        for (int n = 0; n < 2 * C::NP; ++n)
          *reinterpret_cast<uint32_t*>(orow + n * 8) = pack_bf16(o[n][2 * h] * inv[h], o[n][2 * h + 1] * inv[h]);
      }
      continue;
    }
    const int r = pc.r;
    const long long seg = (long long)c + r;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float* orow = p.o_part + (seg * C::HG + head_l0 + h * 8) * LAT + j * C::DIMW + (lane & 3) * 2;
#pragma unroll
      for (int n = 0; n < 2 * C::NP; ++n)
        *reinterpret_cast<float2*>(orow + n * 8) = make_float2(o[n][2 * h] * inv[h], o[n][2 * h + 1] * inv[h]);
      if (j == 0 && (lane & 3) == 0) p.lse_part[seg * C::HG + head_l0 + h * 8] = lse[h];
    }
    __threadfence();
    cbar(C::CT);
    const int c_first = cta_of(pc.row_w0, W, G);
    const int c_last = cta_of(pc.row_w0 + pc.n - 1, W, G);
    if (tid == 0) {
      const int prev = atomicAdd(p.counters + r, 1);
      const bool last = prev == c_last - c_first;
      if (last) p.counters[r] = 0;  // every segment has arrived: ready for the next launch
      *s_flag = last ? 1 : 0;
    }
    cbar(C::CT);
    if (*s_flag) {
      // Merge the row's segments (written by CTAs c_first..c_last, read from L2). The
      // merge sits at the end of some CTA's range, so it is built for latency: one
      // pass of online log-sum-exp per head (all heads at once), then one batch of
      // independent loads per segment for every thread's 16 (head, 4-dim) items.
      __threadfence();
      if (tid == 0) sk_mark(p, 60);
      if (tid < C::HG) {
        float M = -INFINITY, S = 0.f;
#pragma unroll 4
        for (int cc = c_first; cc <= c_last; ++cc) {
          const float l = __ldcg(p.lse_part + ((long long)cc + r) * C::HG + tid);
          if (l == -INFINITY) continue;
          const float mn = fmaxf(M, l);
          S = S * fast_exp2(M - mn) + fast_exp2(l - mn);
          M = mn;
        }
        sM[tid] = M;
        sS[tid] = S > 0.f ? 1.f / S : 0.f;
      }
      cbar(C::CT);
      const int d = (tid & 127) * 4, h0 = tid >> 7;  // heads h0 + k * HT, k < 16
      float acc[16][4];
#pragma unroll
      for (int k = 0; k < 16; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
      for (int cc = c_first; cc <= c_last; ++cc) {
        const long long sg = (long long)cc + r;
        float l[16];
        float4 v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int h = h0 + k * HT;
          l[k] = __ldcg(p.lse_part + sg * C::HG + h);
          v[k] = __ldcg(reinterpret_cast<const float4*>(p.o_part + (sg * C::HG + h) * LAT + d));
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int h = h0 + k * HT;
          const float wt = (l[k] == -INFINITY) ? 0.f : fast_exp2(l[k] - sM[h]) * sS[h];
          acc[k][0] += wt * v[k].x; acc[k][1] += wt * v[k].y; acc[k][2] += wt * v[k].z; acc[k][3] += wt * v[k].w;
        }
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int h = h0 + k * HT;
        bf16* orow = p.out + ((long long)pc.b * p.H + pc.g * C::HG + h) * LAT + d;
        *reinterpret_cast<uint2*>(orow) = make_uint2(pack_bf16(acc[k][0], acc[k][1]), pack_bf16(acc[k][2], acc[k][3]));
      }
      if (tid == 0) sk_mark(p, 61);
    }
    cbar(C::CT);  // s_flag and the statistics are rewritten by the next piece
  }
  if (!ok) return;
  if (tid == 0) sk_mark(p, 63);
  // sequences without context: zero output, written by CTA (b mod grid)
  for (int b = c; b < B; b += gridDim.x) {
    if (sW[b + 1] != sW[b]) continue;
    for (int e = tid; e < p.H * (LAT / 8); e += C::CT)
      *reinterpret_cast<uint4*>(p.out + ((long long)b * p.H) * LAT + e * 8) = make_uint4(0, 0, 0, 0);
  }
}

template <int HT, int MINB>
void launch(const MlaDecodeLaunch& l, int num_sms) {
  using C = Cfg<HT, MINB>;
  CUtensorMap tq, tkv;
  make_tmap_2d(&tq, l.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (long long)l.B * l.H, DIM, DIM, C::HG, 64);
  make_tmap_2d(&tkv, l.cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.num_slots, DIM, DIM, TOK, 64);
  auto kern = mla_decode_sk_kernel<HT, MINB>;
  set_smem_bytes(kern, C::SMEM);
  Params p;
  p.block_table = l.block_table;
  p.max_blocks = l.max_blocks;
  p.context_lens = l.context_lens;
  p.out = static_cast<bf16*>(l.out);
  p.o_part = l.o_part;
  p.lse_part = l.lse_part;
  p.counters = l.counters;
  p.B = l.B;
  p.H = l.H;
  p.NG = l.H / C::HG;
  p.scale_log2 = l.scale * 1.4426950408889634f;
  p.early = l.early;
  p.err = l.err;
  p.trace = l.trace;
  launch_k(kern, dim3(num_sms * MINB), dim3(C::THREADS), C::SMEM, l.stream, tq, tkv, p);
}

// CTAs per SM of the 16-head kernel: 2 (two stages each, default) or 1 (five stages;
// SPARKPIPE_MLA_SK_CTAS=1).
int ctas_16() {
  static const int v = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_SK_CTAS");
    return (e && e[0] == '1') ? 1 : 2;
  }();
  return v;
}

}  // namespace mlask

int mla_sk_heads_per_cta(int heads) {
  if (heads == 16) return 16;
  if (heads % 32 == 0) return 32;
  return 0;
}

bool mla_sk_supported(int B, int H) { return B >= 1 && B <= mlask::MAX_B && mla_sk_heads_per_cta(H) > 0; }

long long mla_sk_segments(int B, int H, int num_sms) {
  const int hg = mla_sk_heads_per_cta(H);
  const int ctas = num_sms * (hg == 16 ? mlask::ctas_16() : 1);
  return hg ? (long long)ctas + (long long)(H / hg) * B : 0;
}

void mla_decode_sk(const MlaDecodeLaunch& l, int num_sms) {
  if (l.B <= 0) return;
  if (!mla_sk_supported(l.B, l.H)) throw std::runtime_error("mla_decode_sk: unsupported batch / head count");
  if (l.kv_lora != mlask::LAT || l.rope != 64 || l.block_size != mlask::BLK)
    throw std::runtime_error("mla_decode_sk: supports kv_lora 512, rope 64, 64-token blocks");
  if (!l.o_part || !l.lse_part || !l.counters) throw std::runtime_error("mla_decode_sk: scratch missing");
  if (mla_sk_heads_per_cta(l.H) == 16) {
    if (mlask::ctas_16() == 2) mlask::launch<1, 2>(l, num_sms);
    else mlask::launch<1, 1>(l, num_sms);
  } else {
    mlask::launch<2, 1>(l, num_sms);
  }
}

void kernel_attrs_mla_sk(std::vector<KernelAttr>& out) {
  push_kernel_attr(out, "mla_decode_sk_kernel<1,2>", mlask::mla_decode_sk_kernel<1, 2>);
  push_kernel_attr(out, "mla_decode_sk_kernel<1,1>", mlask::mla_decode_sk_kernel<1, 1>);
  push_kernel_attr(out, "mla_decode_sk_kernel<2,1>", mlask::mla_decode_sk_kernel<2, 1>);
}

}  // namespace sp
