// Chunked / paged MLA prefill attention on the 5th-generation tensor cores
// (tcgen05), sm_100a. Same contract as prefill_attn.cu (expanded form: per-head
// q_nope/k_nope 128, shared rope key 64, v 128; variable-length batches; query i
// of a chunk of Lq against Lk keys sees keys j <= Lk - Lq + i).
//
// One CTA = 128 queries of one head. Per 128-key tile:
//
//   S[128 q, 128 k]  = Q[128, 192] . K_tile[128, 192]^T   (12 x tcgen05.mma M=128 N=128 K=16)
//   O[128 q, 128 d] += P[128, 128] . V_tile[128, 128]      ( 8 x tcgen05.mma M=128 N=128 K=16)
//
// S and O accumulate in tensor memory (two S buffers, O), and P is written back
// into tensor memory (two buffers, bf16 pairs per column) as the A operand of the
// second product, so it costs no shared memory: Q (three 64-dim boxes, 48 KB) and
// a double-buffered 80 KB stage of K (two nope boxes + the rope box) and V (two
// boxes) fit. V is the B operand of the second product read MN-major (keys are
// its K). 64-key tiles with P in shared memory measured 800 TFLOP/s.
//
// A query row's TMEM data-path lane belongs to two softmax threads (warps w and
// w + 4), each reading half of the row of S: they mask, take the half-row max,
// agree on the row max through shared memory, exponentiate, keep their own partial
// sums and store their half of the row of P into tensor memory. One warp per sub-partition left the tensor
// pipe idle two thirds of the time (the softmax latency per tile). The running max is lazy: P is taken against the current max unless the
// row's tile max exceeds it by more than 2^8; only then (warp-uniformly) is the
// row's O rescaled in TMEM, after the previous tile's second product finished.
//
// Warp roles (320 threads): warps 0-7 softmax / epilogue (two per TMEM lane
// quadrant, each owning half of its query rows), warp 8 TMA producer, warp 9
// tensor-core issue (one thread, never blocking on one product while the other
// could go) and TMEM allocation. Barriers that one side may pass twice before
// the other looks are kept per tile parity. Every wait is bounded; on a timeout the
// CTA records the error, drains its copies and MMAs and returns.
//
// Reference: PagedPrefillPlan / BulkPrefillPlan in
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:736-779.
#include <cuda_runtime.h>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "mma_sync.cuh"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace fatc {
constexpr int BM = 128;                  // queries per CTA
constexpr int BN = 128;                  // keys per tile
constexpr int QBOX = BM * 128;           // 128 rows x 64 dims bf16
constexpr int KBOX = BN * 128;           // 128 keys x 64 dims bf16
constexpr int STAGES = 2;
constexpr int STAGE = 5 * KBOX;          // K nope (2) + K rope (1) + V (2): 80 KB
constexpr int OFF_Q = 0;
constexpr int OFF_KV = 3 * QBOX;
constexpr int OFF_XCH = OFF_KV + STAGES * STAGE;  // [2 parity][2 halves][128 rows] half-row maxima
constexpr int OFF_BAR = OFF_XCH + 2 * 2 * BM * 4;
constexpr int NBAR = 16;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
constexpr int S_COL = 0;                 // two S buffers of 128 fp32 columns
constexpr int O_COL = 256;               // O: 128 fp32 columns
constexpr int P_COL = 384;               // two P buffers of 64 columns (128 bf16 keys, packed pairs)
constexpr int TMEM_COLS = 512;
constexpr int SOFTMAX_THREADS = 256;     // 8 warps: two per TMEM lane quadrant, one per half row
constexpr int PRODUCER_WARP = 8, MMA_WARP = 9;
constexpr int THREADS = 320;
constexpr float RESCALE_LOG2 = 8.f;
}  // namespace fatc

struct FaTcParams {
  const int* cu_q;
  const int* cu_k;
  bf16* o;
  long long o_tok, o_head;
  int H, causal;
  int q_x0, k_x0, v_x0;          // x coordinate of head 0 in the q / k / v tensor maps
  int q_xh, k_xh, v_xh;          // x stride per head (elements)
  float scale_log2;
  int* err;
};

// AND of `v` over `n` threads at named barrier `id` (also a memory barrier among them).
SP_DEVI bool named_bar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(fatc::THREADS, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmKpe, const __grid_constant__ CUtensorMap tmV,
                           const FaTcParams p) {
  using namespace fatc;
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.z, h = blockIdx.y;
  const int q_begin = p.cu_q[b], q_len = p.cu_q[b + 1] - q_begin;
  const int k_begin = p.cu_k[b], k_len = p.cu_k[b + 1] - k_begin;
  const int q0 = blockIdx.x * BM;
  if (q0 >= q_len) return;  // uniform over the CTA
  const int diag = k_len - q_len;  // query i sees keys <= diag + i
  const int kend = p.causal ? min(k_len, diag + min(q0 + BM, q_len)) : k_len;
  const int nkt = kend > 0 ? (kend + BN - 1) / BN : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem + OFF_Q);
  const uint32_t sKV = smem_u32(smem + OFF_KV);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full = bars;        // [3] stage landed
  uint64_t* empty = bars + 3;   // [3] second product of the stage's tile done
  uint64_t* sdone = bars + 6;   // [2] S ready, by tile parity
  uint64_t* odone = bars + 8;   // [2] O product of a tile done, by tile parity
  uint64_t* pready = bars + 10; // [2] P written (and O rescaled), by tile parity
  uint64_t* qbar = bars + 12;
  uint64_t* fin = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 14; ++i) mbar_init(&bars[i], (i >= 10 && i < 12) ? SOFTMAX_THREADS : 1);
    *s_err = 0;
    fence_mbarrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc<TMEM_COLS>(tmem_slot);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == PRODUCER_WARP) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && nkt > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmKpe);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(qbar, 3 * QBOX);
      for (int c = 0; c < 3; ++c)
        tma_load_2d(smem + OFF_Q + c * QBOX, &tmQ, qbar, p.q_x0 + h * p.q_xh + c * 64, q_begin + q0);
      int issued = 0;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % STAGES, n = j / STAGES;
        if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, s_err, p.err, kErrWaitTimeoutProducer)) break;
        const int row = k_begin + j * BN;
        uint8_t* st = smem + OFF_KV + s * STAGE;
        mbar_arrive_expect_tx(&full[s], STAGE);
        tma_load_2d(st, &tmK, &full[s], p.k_x0 + h * p.k_xh, row);
        tma_load_2d(st + KBOX, &tmK, &full[s], p.k_x0 + h * p.k_xh + 64, row);
        tma_load_2d(st + 2 * KBOX, &tmKpe, &full[s], 0, row);
        tma_load_2d(st + 3 * KBOX, &tmV, &full[s], p.v_x0 + h * p.v_xh, row);
        tma_load_2d(st + 4 * KBOX, &tmV, &full[s], p.v_x0 + h * p.v_xh + 64, row);
        issued = j + 1;
      }
      if (*s_err != 0) {  // drain this CTA's copies still in flight
        mbar_drain(qbar, 0);
        for (int j = max(0, issued - STAGES); j < issued; ++j) mbar_drain(&full[j % STAGES], (j / STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    // ---------------------------------------------------------------- tensor-core issue
    if (lane == 0 && nkt > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BN);
      constexpr uint32_t idO = idesc_bf16_f32_bmn(BM, 128);
      auto issue_s = [&](int j) {
        const uint32_t st = sKV + (j % STAGES) * STAGE;
        const uint32_t d = tbase + S_COL + (j & 1) * BN;
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(d, sdesc_kmajor_sw128(sQ + c * QBOX + kk * 32), sdesc_kmajor_sw128(st + c * KBOX + kk * 32), idS,
                     (c | kk) != 0);
        umma_commit(&sdone[j & 1]);
      };
      auto issue_o = [&](int j) {
        const uint32_t st = sKV + (j % STAGES) * STAGE;
        const uint32_t pa = tbase + P_COL + (j & 1) * (BN / 2);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)  // A = P from tensor memory: 16 keys = 8 columns
          umma_f16_ts(tbase + O_COL, pa + kk * 8, sdesc_mnmajor_sw128(st + 3 * KBOX + kk * 2048, KBOX), idO,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&odone[j & 1]);
        umma_commit(&empty[j % STAGES]);
      };
      bool ok = mbar_wait(qbar, 0, s_err, p.err, kErrWaitTimeoutMma);
      int ns = 0, no = 0;
      long long t0 = clock64();
      while (ok && no < nkt) {
        bool progressed = false;
        // S of tile ns once its stage landed and the softmax is done with the S buffer
        // it overwrites (the O product of tile ns - 2 was issued)
        if (ns < nkt && ns <= no + 1 && mbar_test_wait(&full[ns % STAGES], (ns / STAGES) & 1)) {
          tc_fence_after();
          issue_s(ns);
          ++ns;
          progressed = true;
        }
        if (no < ns && mbar_test_wait(&pready[no & 1], (no >> 1) & 1)) {
          tc_fence_after();
          issue_o(no);
          ++no;
          progressed = true;
        }
        if (progressed) {
          t0 = clock64();
        } else if (*s_err != 0) {
          ok = false;
        } else if (clock64() - t0 > kWaitBudgetCycles) {
          *s_err = kErrWaitTimeoutMma;
          atomicCAS(p.err, 0, kErrWaitTimeoutMma);
          ok = false;
        }
      }
      umma_commit(fin);
      mbar_drain(fin, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps 0-7
    // Warps w and w + 4 share TMEM lane quadrant w % 4: each thread owns half of its
    // query row (keys [32 hf, 32 hf + 32) of a tile, O columns [64 hf, 64 hf + 64)).
    // The halves agree on the row max through shared memory at the per-tile barrier,
    // which is also where all 256 threads agree whether every wait succeeded (a
    // thread never leaves the loop alone, so nobody is left at the barrier).
    const int quad = warp & 3, hf = warp >> 2;
    const int r = quad * 32 + lane;    // query row of the tile = TMEM lane
    const int qi = q0 + r;
    const int limit = qi < q_len ? (p.causal ? min(k_len, diag + qi + 1) : k_len) : 0;  // keys [0, limit)
    const uint32_t t_lane = tbase + (uint32_t(quad * 32) << 16);
    float* xch = reinterpret_cast<float*>(smem + OFF_XCH);
    float m_run = -INFINITY, l_part = 0.f;
    bool ok = true, bad = false;
    for (int j = 0; j < nkt; ++j) {
      bool okl = !bad && mbar_wait(&sdone[j & 1], (j >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue);
      constexpr int HK = BN / 2;  // keys per half row
      float sv[HK];
      float mh = -INFINITY;
      const int kb = j * BN + hf * HK;
      if (okl) {
        tc_fence_after();
        uint32_t a[4][16];
        const uint32_t ta = t_lane + S_COL + (j & 1) * BN + hf * HK;
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld16_issue(ta + q * 16, a[q]);
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld_wait(a[q]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int c = 0; c < 16; ++c) sv[q * 16 + c] = __uint_as_float(a[q][c]);
        if (kb + HK > limit) {  // half tile crosses the row's key limit
#pragma unroll
          for (int c = 0; c < HK; ++c)
            if (kb + c >= limit) sv[c] = -INFINITY;
        }
        float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int c = 4; c < HK; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
        mh = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      // the P buffer of this parity was read by the O product of two tiles back
      if (okl && j >= 2) okl = mbar_wait(&odone[j & 1], ((j - 2) >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue);
      float* xj = xch + (j & 1) * 2 * BM;
      xj[hf * BM + r] = mh;
      ok = named_bar_and(1, SOFTMAX_THREADS, okl);
      if (!ok) break;
      const float mt = fmaxf(mh, xj[(1 - hf) * BM + r]) * p.scale_log2;  // scale > 0
      const bool need = mt > m_run + fatc::RESCALE_LOG2;  // the same in both halves of the row
      if (__any_sync(0xffffffffu, need)) {
        float alpha = 1.f;
        if (need) {
          alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mt);
          m_run = mt;
          l_part *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          // O holds tiles 0 .. j-1 once the previous O product is done; this thread
          // rescales its half of the row
          const bool okw = __all_sync(0xffffffffu, mbar_wait(&odone[(j - 1) & 1], ((j - 1) >> 1) & 1, s_err, p.err,
                                                              kErrWaitTimeoutEpilogue));
          if (okw) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 64; c += 16) {
              float v[16];
              tmem_ld16(t_lane + O_COL + hf * 64 + c, v);
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] *= alpha;
              tmem_st16(t_lane + O_COL + hf * 64 + c, v);
            }
          } else {
            bad = true;  // reported at the next tile's barrier
          }
        }
      }
      // P = 2^(s * scale - m) as bf16 (masked scores are -inf: 2^-inf = 0; a row with
      // no key yet uses m = 0), this half row's 32 columns of the P buffer in TMEM
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = fast_exp2(fmaf(sv[q * 32 + 2 * e], p.scale_log2, neg_m));
          const float bq = fast_exp2(fmaf(sv[q * 32 + 2 * e + 1], p.scale_log2, neg_m));
          ls[e & 3] += a + bq;
          w[e] = __uint_as_float(pack_bf16(a, bq));
        }
        tmem_st16(t_lane + P_COL + (j & 1) * (BN / 2) + hf * (HK / 2) + q * 16, w);
      }
      l_part += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tc_fence_before();
      mbar_arrive(&pready[j & 1]);
    }
    if (ok) {
      const bool okl = !bad && (nkt == 0 || mbar_wait(&odone[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1, s_err, p.err,
                                                       kErrWaitTimeoutEpilogue));
      // the exchange slots of tile nkt - 2's parity: their readers all passed tile nkt - 1's barrier
      float* xl = xch + (nkt & 1) * 2 * BM;
      xl[hf * BM + r] = l_part;
      ok = named_bar_and(1, SOFTMAX_THREADS, okl);
    }
    if (ok) {
      tc_fence_after();
      const float* xl = xch + (nkt & 1) * 2 * BM;
      const float l = xl[r] + xl[BM + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.o + (long long)(q_begin + qi) * p.o_tok + (long long)h * p.o_head + hf * 64;
#pragma unroll 1
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        if (nkt > 0) {
          tmem_ld16(t_lane + O_COL + hf * 64 + c, v);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = 0.f;
        }
        if (qi < q_len) {
          uint4 w0 = make_uint4(pack_bf16(v[0] * inv, v[1] * inv), pack_bf16(v[2] * inv, v[3] * inv),
                                pack_bf16(v[4] * inv, v[5] * inv), pack_bf16(v[6] * inv, v[7] * inv));
          uint4 w1 = make_uint4(pack_bf16(v[8] * inv, v[9] * inv), pack_bf16(v[10] * inv, v[11] * inv),
                                pack_bf16(v[12] * inv, v[13] * inv), pack_bf16(v[14] * inv, v[15] * inv));
          *reinterpret_cast<uint4*>(orow + c) = w0;
          *reinterpret_cast<uint4*>(orow + c + 8) = w1;
        }
      }
    }
  }
  __syncthreads();
  if (warp == fatc::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc<fatc::TMEM_COLS>(tbase);
  }
}

// TMA needs 16-byte aligned bases and row strides and head offsets that keep every
// box's x coordinate a multiple of 8 elements; otherwise the mma.sync kernel runs.
bool prefill_attention_tc_ok(const PrefillAttnLaunch& l) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  return al(l.q) && al(l.k) && al(l.kpe) && al(l.v) && al(l.o) && l.q_tok % 8 == 0 && l.k_tok % 8 == 0 &&
         l.kpe_tok % 8 == 0 && l.v_tok % 8 == 0 && l.q_head % 8 == 0 && l.k_head % 8 == 0 && l.v_head % 8 == 0 &&
         l.o_tok % 8 == 0 && l.o_head % 8 == 0 && l.q_rows > 0 && l.k_rows > 0;
}

void prefill_attention_tc(const PrefillAttnLaunch& l) {
  using namespace fatc;
  CUtensorMap tq, tk, tkpe, tv;
  // each map starts at the tensor's base and spans every head's columns of a row
  const long long qcols = (long long)(l.H - 1) * l.q_head + 192;
  const long long kcols = (long long)(l.H - 1) * l.k_head + 128;
  const long long vcols = (long long)(l.H - 1) * l.v_head + 128;
  make_tmap_2d(&tq, l.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.q_rows, qcols, l.q_tok, BM, 64);
  make_tmap_2d(&tk, l.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.k_rows, kcols, l.k_tok, BN, 64);
  make_tmap_2d(&tkpe, l.kpe, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.k_rows, 64, l.kpe_tok, BN, 64);
  make_tmap_2d(&tv, l.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.k_rows, vcols, l.v_tok, BN, 64);
  set_smem_bytes(prefill_attn_tc_kernel, SMEM);
  FaTcParams p;
  p.cu_q = l.cu_q;
  p.cu_k = l.cu_k;
  p.o = (bf16*)l.o;
  p.o_tok = l.o_tok;
  p.o_head = l.o_head;
  p.H = l.H;
  p.causal = l.causal;
  p.q_x0 = 0;
  p.k_x0 = 0;
  p.v_x0 = 0;
  p.q_xh = (int)l.q_head;
  p.k_xh = (int)l.k_head;
  p.v_xh = (int)l.v_head;
  p.scale_log2 = l.scale * 1.4426950408889634f;
  p.err = l.err;
  if (l.B > 65535 || l.H > 65535) throw std::runtime_error("prefill_attention: grid limits");
  dim3 grid((l.max_q + BM - 1) / BM, l.H, l.B);
  launch_k(prefill_attn_tc_kernel, grid, dim3(THREADS), SMEM, l.stream, tq, tk, tkpe, tv, p);
}

void kernel_attrs_prefill(std::vector<KernelAttr>& out) {
  push_kernel_attr(out, "prefill_attn_tc_kernel", prefill_attn_tc_kernel);
}

}  // namespace sp
