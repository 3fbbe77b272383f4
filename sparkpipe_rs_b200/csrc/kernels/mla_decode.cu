// MLA paged latent-KV decode attention (absorbed form), sm_100a.
//
// For each sequence b and head h:  o[b,h,:] = softmax(scale * q[b,h,:] . K^T) V
// where K = cache rows [latent (kv_lora) | rope key (rope)] of the sequence's
// paged blocks and V = the latent part of the same rows. All heads of a head
// group share every KV byte, so one CTA streams each KV stage once (TMA,
// 128-byte swizzled sub-tiles, double buffered) and all of its warps consume it.
//
// Stages hold TOK tokens: 64 (one whole cache block, 74 KB per stage, one CTA per
// SM; the default) or 32 (half a cache block, 37 KB per stage, two CTAs per SM).
//
// Head groups of one (sequence, split) are adjacent in the grid (blockIdx.x), so
// with more heads than one CTA holds (64 heads = 2 groups of 32) the groups stream
// the same KV blocks at about the same time and the second read hits L2.
//
// Warp layout: NJ warps per 16-head tile. For each stage a warp computes the
// scores of TOK/NJ tokens and the output of 512/NJ latent dims, so NJ = 8 halves
// the serial mma.sync work per warp; measured on 16-head decode (B=64, ctx 1024)
// it was 6% slower than NJ = 4, so both widths use 4.
//
// Two kernels: the mma.sync one described here (the default) and a tcgen05 one
// further down (tensor-memory accumulators; selected with impl = MLA_IMPL_TC or
// SPARKPIPE_MLA_KERNEL=tc). Both share the split-KV scratch format and combine.
//
// Split-KV: a sequence's blocks are divided over `splits` CTAs; each writes a
// normalised partial output and its log-sum-exp, and a combine kernel merges
// them. With splits == 1 the kernel writes the bf16 output directly.
//
// Reference: PHASE_MLA_ATTENTION with ABSORBED_LATENT mode and block tables in
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:445-460,
// 563-568 and the pipeline-slot buffers :815-867.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"
#include "mma_sync.cuh"

namespace sp {

using bf16 = __nv_bfloat16;

struct MlaKParams {
  const int* block_table;
  int max_blocks;
  const int* context_lens;
  bf16* out;
  float* o_part;
  float* lse_part;
  int B, H, splits;
  float scale_log2;
  int* err;
  unsigned long long* trace;  // tcgen05 kernel: event times of CTA (0,0,0), or null
  // mma.sync kernel: when set, row b's last context token is read from cache row
  // last_slot[b] instead of its block-table position (the alternate leaves of a
  // tree verify, whose KV sits in a shadow slot)
  const int* last_slot;
  const bf16* cache;
};

constexpr int MLA_DIM = 576;     // kv_lora 512 + rope 64
constexpr int MLA_LAT = 512;
constexpr int MLA_CHUNKS = 9;    // 64-element (128-byte) column chunks
constexpr int MLA_BLK = 64;      // tokens per cache block

template <int HG, int NJ, int TOK, int NST = 2>
struct MlaCfg {
  static constexpr int STAGES = NST;  // KV stages in flight
  static constexpr int WARPS = NJ * (HG / 16);
  static constexpr int STAGE_BYTES = MLA_CHUNKS * TOK * 128;
  static constexpr int PER_BLOCK = MLA_BLK / TOK;  // stages per cache block
  static constexpr int TOKW = TOK / NJ;       // tokens per warp in S = Q K^T
  static constexpr int NT = TOKW / 8;         // n8 tiles per warp in S
  static constexpr int DIMW = MLA_LAT / NJ;   // latent dims per warp in O = P V
  static constexpr int NP = DIMW / 16;        // n8-tile pairs per warp in O
  static constexpr int Q_BYTES = MLA_CHUNKS * HG * 128;
  static constexpr int P_PITCH = TOK + 8;     // bf16 elements per P row (padded)
  static constexpr int OFF_KV = (Q_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_P = OFF_KV + NST * STAGE_BYTES;
  static constexpr int OFF_STAT = OFF_P + HG * P_PITCH * 2;
  static constexpr int OFF_BAR = OFF_STAT + 2 * NJ * HG * 4;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;
  static constexpr int MIN_CTAS = (2 * SMEM <= 227 * 1024) ? 2 : 1;
};

// SPLIT: the S = Q K^T product of a warp accumulates even and odd 16-wide K steps
// into two register sets (two dependency chains of 18 MMAs instead of one of 36),
// summed before the softmax.
template <int HG, int NJ, int TOK, bool LAST = false, bool SPLIT = false, int NST = 2>
__global__ void __launch_bounds__(MlaCfg<HG, NJ, TOK, NST>::WARPS * 32, MlaCfg<HG, NJ, TOK, NST>::MIN_CTAS)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                      const MlaKParams p) {
  griddep_wait();
  griddep_launch();
  using C = MlaCfg<HG, NJ, TOK, NST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = smem_u32(smem + C::OFF_KV);
  bf16* sP = reinterpret_cast<bf16*>(smem + C::OFF_P);
  float* sMax = reinterpret_cast<float*>(smem + C::OFF_STAT);  // [NJ][HG]
  float* sSum = sMax + NJ * HG;                                 // [NJ][HG]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* qbar = full + NST;
  volatile int* s_err = reinterpret_cast<volatile int*>(qbar + 1);

  const int hg = blockIdx.x;
  const int b = blockIdx.y;
  const int split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = warp / NJ, j = warp % NJ;

  const int ctx = p.context_lens[b];
  const int nblk = (ctx + MLA_BLK - 1) / MLA_BLK;
  const int per = (nblk + p.splits - 1) / p.splits;
  const int kb0 = min(nblk, split * per);
  const int kb1 = min(nblk, kb0 + per);
  // stages of this split: PER_BLOCK per cache block, none past the context
  const int nb = max(0, min((kb1 - kb0) * C::PER_BLOCK, (ctx - kb0 * MLA_BLK + TOK - 1) / TOK));
  const int* bt = p.block_table + (long long)b * p.max_blocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) mbar_init(&full[i], 1);
    mbar_init(qbar, 1);
    *s_err = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmKV);
  }
  __syncthreads();

  auto issue_block = [&](int i) {  // thread 0 only; stage i = part (i % PER_BLOCK) of block kb0 + i / PER_BLOCK
    const int s = i % NST;
    const int pb = bt[kb0 + i / C::PER_BLOCK];
    const int row = pb * MLA_BLK + (i % C::PER_BLOCK) * TOK;
    uint64_t* bar = &full[s];
    mbar_arrive_expect_tx(bar, C::STAGE_BYTES);
    uint8_t* dst = smem + C::OFF_KV + s * C::STAGE_BYTES;
#pragma unroll 1
    for (int c = 0; c < MLA_CHUNKS; ++c) tma_load_2d(dst + c * TOK * 128, &tmKV, bar, c * 64, row);
  };
  int issued = 0;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmKV);
    mbar_arrive_expect_tx(qbar, C::Q_BYTES);
    for (int c = 0; c < MLA_CHUNKS; ++c) tma_load_2d(smem + c * HG * 128, &tmQ, qbar, c * 64, b * p.H + hg * HG);
    for (; issued < NST && issued < nb; ++issued) issue_block(issued);
  }

  float o[2 * C::NP][4];
#pragma unroll
  for (int n = 0; n < 2 * C::NP; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int r_lo = lane >> 2;           // fragment rows r_lo and r_lo + 8
  const int qrow = mt * 16;

  bool ok = mbar_wait(qbar, 0, s_err, p.err, kErrWaitTimeoutMma);
  ok = __syncthreads_and(ok);
  for (int i = 0; ok && i < nb; ++i) {
    const int s = i % NST;
    bool got = mbar_wait(&full[s], (i / NST) & 1, s_err, p.err, kErrWaitTimeoutMma);
    if (!__syncthreads_and(got)) { ok = false; break; }
    const uint32_t kvb = sKV + s * C::STAGE_BYTES;
    if constexpr (LAST) {
      const int t_last = ctx - 1, t0 = kb0 * MLA_BLK + i * TOK;
      const int src = p.last_slot[b];
      if (t_last >= t0 && t_last < t0 + TOK && src >= 0 &&
          src != bt[t_last / MLA_BLK] * MLA_BLK + t_last % MLA_BLK) {  // block-uniform
        // overwrite the stage's row of that token (128-byte swizzled, 16-byte units)
        const int tr = t_last - t0;
        uint8_t* st = smem + C::OFF_KV + s * C::STAGE_BYTES;
        for (int e = threadIdx.x; e < MLA_CHUNKS * 8; e += blockDim.x) {
          const int c = e >> 3, u = e & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(p.cache + (long long)src * MLA_DIM + c * 64 + u * 8);
          *reinterpret_cast<uint4*>(st + c * TOK * 128 + tr * 128 + ((u ^ (tr & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();  // the next TMA write of this stage is ordered after these
        __syncthreads();
      }
    }

    // ---- S = Q K^T for 16 heads x TOKW tokens of this warp
    float sc[C::NT][4], sc2[C::NT][4];
#pragma unroll
    for (int n = 0; n < C::NT; ++n) {
      sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      sc2[n][0] = sc2[n][1] = sc2[n][2] = sc2[n][3] = 0.f;
    }
#pragma unroll 4
    for (int kk = 0; kk < MLA_DIM / 16; ++kk) {
      const int c = kk >> 2;
      const int cc = (kk & 3) * 16;
      uint32_t a[4];
      ldsm_x4(a, swz128(sQ + c * HG * 128, qrow + (lane & 15), cc + (lane >> 4) * 8));
      float (*acc)[4] = (SPLIT && (kk & 1)) ? sc2 : sc;
      if constexpr (C::NT == 2) {
        uint32_t bb[4];
        ldsm_x4(bb, swz128(kvb + c * TOK * 128, j * 16 + (lane & 7) + (lane >> 4) * 8, cc + ((lane >> 3) & 1) * 8));
        mma16816(acc[0], a, bb[0], bb[1]);
        mma16816(acc[1], a, bb[2], bb[3]);
      } else {
        uint32_t bb[2];
        ldsm_x2(bb, swz128(kvb + c * TOK * 128, j * 8 + (lane & 7), cc + ((lane >> 3) & 1) * 8));
        mma16816(acc[0], a, bb[0], bb[1]);
      }
    }
    if constexpr (SPLIT) {
#pragma unroll
      for (int n = 0; n < C::NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[n][e] += sc2[n][e];
    }
    // ---- scale, mask, row max
    const int tok0 = kb0 * MLA_BLK + i * TOK + j * C::TOKW;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < C::NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tok0 + n * 8 + (lane & 3) * 2 + (e & 1);
        float v = sc[n][e] * p.scale_log2;
        if (tok >= ctx) v = -INFINITY;
        sc[n][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    if ((lane & 3) == 0) {
      sMax[j * HG + qrow + r_lo] = mx[0];
      sMax[j * HG + qrow + r_lo + 8] = mx[1];
    }
    __syncthreads();
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = qrow + r_lo + h * 8;
      float mn = m_run[h];
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) mn = fmaxf(mn, sMax[jj * HG + row]);
      alpha[h] = (m_run[h] == -INFINITY) ? 0.f : exp2f(m_run[h] - mn);
      m_run[h] = mn;
      l_run[h] *= alpha[h];
    }
    // ---- P = exp2(S - m), stored bf16 for the PV product
#pragma unroll
    for (int n = 0; n < C::NT; ++n) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mrow = m_run[e >> 1];
        pv[e] = (sc[n][e] == -INFINITY) ? 0.f : exp2f(sc[n][e] - mrow);
        l_run[e >> 1] += pv[e];
      }
      const int col = j * C::TOKW + n * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(sP + (qrow + r_lo) * C::P_PITCH + col) = pack_bf16(pv[0], pv[1]);
      *reinterpret_cast<uint32_t*>(sP + (qrow + r_lo + 8) * C::P_PITCH + col) = pack_bf16(pv[2], pv[3]);
    }
#pragma unroll
    for (int n = 0; n < 2 * C::NP; ++n) {
      o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
      o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
    }
    __syncthreads();
    // ---- O[16 heads, DIMW dims of slice j] += P[16, TOK] V[TOK, DIMW]
    const uint32_t sPa = smem_u32(sP);
#pragma unroll
    for (int kk = 0; kk < TOK / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sPa + ((qrow + (lane & 15)) * C::P_PITCH + kk * 16 + (lane >> 4) * 8) * 2);
      const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int np = 0; np < C::NP; ++np) {
        const int dim = j * C::DIMW + np * 16 + (lane >> 4) * 8;
        uint32_t bb[4];
        ldsm_x4_t(bb, swz128(kvb + (dim >> 6) * TOK * 128, tok, dim & 63));
        mma16816(o[2 * np], a, bb[0], bb[1]);
        mma16816(o[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && issued < nb) { issue_block(issued); ++issued; }
  }

  if (!ok) {
    // Drain loads still in flight before the CTA's shared memory is released.
    if (threadIdx.x == 0) {
      for (int i2 = max(0, issued - NST); i2 < issued; ++i2)
        mbar_wait(&full[i2 % NST], (i2 / NST) & 1, s_err, nullptr, 0);
    }
    return;
  }

  // ---- final row sums across the 4 warps of this head tile
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  if ((lane & 3) == 0) {
    sSum[j * HG + qrow + r_lo] = l_run[0];
    sSum[j * HG + qrow + r_lo + 8] = l_run[1];
  }
  __syncthreads();
  float inv[2], lse[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = qrow + r_lo + h * 8;
    float l = 0.f;
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) l += sSum[jj * HG + row];
    inv[h] = l > 0.f ? 1.f / l : 0.f;
    lse[h] = l > 0.f ? m_run[h] + __log2f(l) : -INFINITY;
  }
  const int head0 = hg * HG + qrow + r_lo;
  if (p.splits == 1) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      bf16* orow = p.out + ((long long)b * p.H + head0 + h * 8) * MLA_LAT + j * C::DIMW + (lane & 3) * 2;
#pragma unroll
      for (int n = 0; n < 2 * C::NP; ++n)
        *reinterpret_cast<uint32_t*>(orow + n * 8) = pack_bf16(o[n][2 * h] * inv[h], o[n][2 * h + 1] * inv[h]);
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const long long rowi = ((long long)b * p.splits + split) * p.H + head0 + h * 8;
      float* orow = p.o_part + rowi * MLA_LAT + j * C::DIMW + (lane & 3) * 2;
#pragma unroll
      for (int n = 0; n < 2 * C::NP; ++n)
        *reinterpret_cast<float2*>(orow + n * 8) = make_float2(o[n][2 * h] * inv[h], o[n][2 * h + 1] * inv[h]);
      if (j == 0 && (lane & 3) == 0) p.lse_part[rowi] = lse[h];
    }
  }
}

__global__ void mla_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ lse,
                                   bf16* __restrict__ out, int H, int S) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[((long long)b * S + s) * H + h]);
  float wsum = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int d = threadIdx.x * 4;
  for (int s = 0; s < S; ++s) {
    const float l = lse[((long long)b * S + s) * H + h];
    const float w = (l == -INFINITY) ? 0.f : exp2f(l - M);
    wsum += w;
    if (w > 0.f) {
      const float4 v = *reinterpret_cast<const float4*>(o_part + (((long long)b * S + s) * H + h) * MLA_LAT + d);
      acc[0] += w * v.x; acc[1] += w * v.y; acc[2] += w * v.z; acc[3] += w * v.w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  bf16* orow = out + ((long long)b * H + h) * MLA_LAT + d;
  *reinterpret_cast<uint32_t*>(orow) = pack_bf16(acc[0] * inv, acc[1] * inv);
  *reinterpret_cast<uint32_t*>(orow + 2) = pack_bf16(acc[2] * inv, acc[3] * inv);
}

void mla_combine(const float* o_part, const float* lse_part, void* out, int B, int H, int splits, cudaStream_t s) {
  launch_k(mla_combine_kernel, dim3(B * H), dim3(MLA_LAT / 4), 0, s, o_part, lse_part, (bf16*)out, H, splits);
}

// ============================================================================
// tcgen05 version. One CTA per (head group of HG heads, sequence, KV split), as
// above, but the two products run on the 5th-generation tensor cores with the
// accumulators in tensor memory, the KV tile oriented as the M operand:
//
//   S^T[64 tokens, HG heads] = K_tile[64, 576] . Q[HG, 576]^T          (M = 64)
//   O^T[512 dims, HG heads] += V_tile^T[512, 64] . P^T[HG, 64]^T       (4 x M = 128)
//
// The same 128-byte-swizzled KV stage (nine 64-token x 64-dim TMA boxes) is the
// K-major A operand of the first product and, read through an MN-major
// descriptor, the A operand V^T of the second; only the latent dims (boxes 0-7)
// enter the second. S^T lands with token r in TMEM lane (r % 16) + 32 (r / 16)
// (the M = 64 data-path layout), so each of the 4 softmax warps holds 16 tokens
// x HG heads. The running sums stay per thread and are reduced once at the end.
// The running max is lazy: a tile's scores are exponentiated against the current
// max unless some score exceeds it by more than 2^8 (one vote over the 128
// threads); only then is the max reduced across the 64 token lanes and O^T and the
// sums rescaled (the first tile always sets it). P then stays below 2^8, exact
// enough in bf16, and the common path has no tensor-memory round trip and no
// wait on the previous tile's second product. P^T is written bf16 into a K-major
// swizzled tile (the B operand), double buffered.
//
// Warp roles (192 threads): warps 0-3 softmax / epilogue, warp 4 TMA producer
// (double-buffered 72 KB stages), warp 5 tensor-core issue (one thread) and TMEM
// allocation. The issuing thread never blocks on one product while the other
// could go: the next tile's S^T product (into the other of two S^T buffers) is
// issued as soon as its stage lands, the current tile's O^T product as soon as
// its P^T is written. Barriers that one side may pass twice before the other
// looks are kept per tile parity. Every wait is bounded; on a timeout the CTA
// records the error, drains its copies and MMAs and returns.
namespace mtc {
constexpr int TOK = 64;                       // tokens per stage = one cache block
constexpr int BOX_BYTES = TOK * 128;          // 64 tokens x 64 dims bf16
constexpr int STAGE_BYTES = MLA_CHUNKS * BOX_BYTES;
}  // namespace mtc

template <int HG>
struct MtcCfg {
  static constexpr int Q_BYTES = MLA_CHUNKS * HG * 128;
  static constexpr int OFF_KV = (Q_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_P = OFF_KV + 2 * mtc::STAGE_BYTES;
  static constexpr int P_BYTES = HG * 128;    // P^T: HG rows of 64 bf16 tokens
  static constexpr int OFF_RED = OFF_P + 2 * P_BYTES;       // [2][4][HG] per-warp tile maxima
  static constexpr int OFF_LSUM = OFF_RED + 2 * 4 * HG * 4;  // [4][HG] per-warp sums
  static constexpr int OFF_BAR = OFF_LSUM + 4 * HG * 4;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;  // 12 barriers + TMEM slot + error word
  // S^T accumulation chains (summed when read). Four independent chains measured
  // no faster than one: the cost is per instruction, not the accumulator dependency.
  static constexpr int SCH = 1;
  static constexpr int S_COL = 0;             // two S^T buffers of SCH x HG columns
  static constexpr int O_COL = 2 * SCH * HG;  // O^T: four 128-dim blocks of HG columns
  static constexpr int TMEM_COLS = (O_COL + 4 * HG <= 256) ? 256 : 512;
  static constexpr int THREADS = 192;
};

// AND of `v` over the 128 threads of the softmax warps (named barrier 1).
SP_DEVI bool softmax_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}
SP_DEVI bool softmax_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}
SP_DEVI void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
constexpr float kMlaRescaleLog2 = 8.f;  // lazy max: rescale once a score exceeds it by 2^8

template <int HG>
SP_DEVI void tmem_ld_cols(uint32_t taddr, float (&v)[HG]) {
#pragma unroll
  for (int c = 0; c < HG; c += 16) {
    float t[16];
    tmem_ld16(taddr + c, t);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[c + j] = t[j];
  }
}

// Pipeline event times of the first CTA, for diagnosing the pipeline: trace[ev * 64 + tile].
#define MTC_TRACE(ev, tile)                                                                      \
  do {                                                                                           \
    if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (tile) < 64)          \
      p.trace[(ev) * 64 + (tile)] = globaltimer();                                               \
  } while (0)

template <int HG>
__global__ void __launch_bounds__(192, 1)
    mla_decode_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const MlaKParams p) {
  using C = MtcCfg<HG>;
  griddep_wait();
  griddep_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = smem_u32(smem + C::OFF_KV);
  const uint32_t sP = smem_u32(smem + C::OFF_P);
  float* sRed = reinterpret_cast<float*>(smem + C::OFF_RED);
  float* sLsum = reinterpret_cast<float*>(smem + C::OFF_LSUM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;        // [2] TMA -> MMA
  uint64_t* empty = bars + 2;   // [2] second product done -> stage reusable
  uint64_t* sdone = bars + 4;   // [2] S^T ready
  uint64_t* odone = bars + 6;   // [2] O^T product of a tile done (by tile parity)
  uint64_t* pready = bars + 8;  // [2] softmax wrote P^T (and rescaled O^T), by tile parity
  uint64_t* qbar = bars + 10;
  uint64_t* fin = bars + 11;    // every issued MMA done (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int hg = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = min((p.context_lens[b] + MLA_BLK - 1) / MLA_BLK, p.max_blocks);  // never past the table
  const int ctx = min(p.context_lens[b], nblk * MLA_BLK);
  const int per = (nblk + p.splits - 1) / p.splits;
  const int kb0 = min(nblk, split * per);
  const int nb = max(0, min(nblk, kb0 + per) - kb0);
  const int* bt = p.block_table + (long long)b * p.max_blocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], (i == 8 || i == 9) ? 128 : 1);
    *s_err = 0;
    fence_mbarrier_init();
  }
  if (warp == 5) {
    tmem_alloc<C::TMEM_COLS>(tmem_slot);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (threadIdx.x == 0) MTC_TRACE(5, 0);

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && nb > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      mbar_arrive_expect_tx(qbar, C::Q_BYTES);
      for (int c = 0; c < MLA_CHUNKS; ++c) tma_load_2d(smem + c * HG * 128, &tmQ, qbar, c * 64, b * p.H + hg * HG);
      int issued = 0;
      for (int i = 0; i < nb; ++i) {
        const int s = i & 1;
        if (i >= 2 && !mbar_wait(&empty[s], ((i - 2) >> 1) & 1, s_err, p.err, kErrWaitTimeoutProducer)) break;
        const int row = bt[kb0 + i] * MLA_BLK;
        MTC_TRACE(0, i);
        mbar_arrive_expect_tx(&full[s], mtc::STAGE_BYTES);
        uint8_t* dst = smem + C::OFF_KV + s * mtc::STAGE_BYTES;
#pragma unroll 1
        for (int c = 0; c < MLA_CHUNKS; ++c) tma_load_2d(dst + c * mtc::BOX_BYTES, &tmKV, &full[s], c * 64, row);
        issued = i + 1;
      }
      if (*s_err != 0) {  // drain this CTA's copies still in flight
        mbar_drain(qbar, 0);
        for (int i = max(0, issued - 2); i < issued; ++i) mbar_drain(&full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- tensor-core issue
    if (lane == 0 && nb > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(64, HG);
      constexpr uint32_t idO = idesc_bf16_f32_amn(128, HG);
      auto issue_s = [&](int i) {
        const int s = i & 1;
        const uint32_t kv = sKV + s * mtc::STAGE_BYTES;
#pragma unroll 1
        for (int c = 0; c < MLA_CHUNKS; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // chain kk % SCH
            umma_f16(tbase + C::S_COL + (s * C::SCH + kk % C::SCH) * HG,
                     sdesc_kmajor_sw128(kv + c * mtc::BOX_BYTES + kk * 32),
                     sdesc_kmajor_sw128(sQ + c * HG * 128 + kk * 32), idS, (c * 4 + kk) >= C::SCH);
        umma_commit(&sdone[s]);
      };
      auto issue_o = [&](int i) {
        const int s = i & 1;
        const uint32_t kv = sKV + s * mtc::STAGE_BYTES;
        const uint32_t pb = sP + s * C::P_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int k = 0; k < 4; ++k)  // the four dim blocks are independent accumulators: interleave them
            umma_f16(tbase + C::O_COL + k * HG,
                     sdesc_mnmajor_sw128(kv + 2 * k * mtc::BOX_BYTES + kk * 2048, mtc::BOX_BYTES),
                     sdesc_kmajor_sw128(pb + kk * 32), idO, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&odone[s]);
        umma_commit(&empty[s]);
      };
      // Issue whichever product is ready: S^T of tile ns as soon as its stage has
      // landed (and the softmax is done with the S^T buffer it overwrites, i.e. the
      // second product of tile ns - 2 was issued), O^T of tile no as soon as the
      // softmax has written its P^T. Never block on one while the other could go.
      bool ok = mbar_wait(qbar, 0, s_err, p.err, kErrWaitTimeoutMma);
      int ns = 0, no = 0;
      long long t0 = clock64();
      while (ok && no < nb) {
        bool progressed = false;
        if (ns < nb && ns <= no + 1 && mbar_test_wait(&full[ns & 1], (ns >> 1) & 1)) {
          tc_fence_after();
          MTC_TRACE(1, ns);
          issue_s(ns);
          ++ns;
          progressed = true;
        }
        if (no < ns && mbar_test_wait(&pready[no & 1], (no >> 1) & 1)) {
          tc_fence_after();
          MTC_TRACE(4, no);
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
    // ---------------------------------------------------------------- softmax warps 0-3
    const bool hold = lane < 16;
    const int r = warp * 16 + lane;  // token row of the tile held by this thread (lanes < 16)
    const uint32_t t_lane = tbase + (uint32_t(warp * 32) << 16);
    float m_run[HG], l_part[HG];
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int s = i & 1;
      ok = softmax_bar_and(mbar_wait(&sdone[s], (i >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue));
      if (!ok) break;
      if (threadIdx.x == 0) MTC_TRACE(2, i);
      tc_fence_after();
      float sv[HG];
      tmem_ld_cols<HG>(t_lane + C::S_COL + s * C::SCH * HG, sv);
#pragma unroll
      for (int j = 1; j < C::SCH; ++j) {
        float sj[HG];
        tmem_ld_cols<HG>(t_lane + C::S_COL + (s * C::SCH + j) * HG, sj);
#pragma unroll
        for (int h = 0; h < HG; ++h) sv[h] += sj[h];
      }
      const bool valid = hold && (kb0 + i) * MLA_BLK + r < ctx;
      bool exceed = false;
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        sv[h] = valid ? sv[h] * p.scale_log2 : -INFINITY;
        exceed |= sv[h] > m_run[h] + kMlaRescaleLog2;
      }
      // the P^T buffer of this parity was read by the second product of two tiles back
      const bool pfree = i < 2 || mbar_wait(&odone[s], ((i - 2) >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue);
      if (softmax_bar_or(exceed || !pfree || i == 0)) {
        // slow path, taken by all 128 threads together
        ok = softmax_bar_and(pfree);
        if (!ok) break;
        float mx[HG];
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          float v = sv[h];
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          mx[h] = v;
        }
        float* red = sRed + ((i & 1) * 4 + warp) * HG;
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < HG; h += 4)
            *reinterpret_cast<float4*>(red + h) = make_float4(mx[h], mx[h + 1], mx[h + 2], mx[h + 3]);
        }
        softmax_bar();
        float alpha[HG];
        bool moved = false;
        const float* red0 = sRed + (i & 1) * 4 * HG;
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          const float t = fmaxf(fmaxf(red0[h], red0[HG + h]), fmaxf(red0[2 * HG + h], red0[3 * HG + h]));
          const float mn = fmaxf(m_run[h], t);
          alpha[h] = (mn == m_run[h]) ? 1.f : (m_run[h] == -INFINITY ? 0.f : exp2f(m_run[h] - mn));
          moved |= alpha[h] != 1.f;
          m_run[h] = mn;
          l_part[h] *= alpha[h];
        }
        if (i > 0 && moved) {  // uniform: alpha is the same in every thread
          ok = softmax_bar_and(
              mbar_wait(&odone[(i - 1) & 1], ((i - 1) >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int c = 0; c < HG; c += 16) {
              float v[16];
              const uint32_t ta = t_lane + C::O_COL + k * HG + c;
              tmem_ld16(ta, v);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] *= alpha[c + j];
              tmem_st16(ta, v);
            }
        }
      }
      // P = exp2(S - m) as bf16 into P^T[h][r] (K-major, 128-byte swizzle)
      uint8_t* pbuf = smem + C::OFF_P + s * C::P_BYTES;
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        const float pv = sv[h] == -INFINITY ? 0.f : exp2f(sv[h] - m_run[h]);
        l_part[h] += pv;
        if (hold)
          *reinterpret_cast<bf16*>(pbuf + (h >> 3) * 1024 + (h & 7) * 128 + ((((r >> 3) ^ (h & 7)) & 7) << 4) +
                                   (r & 7) * 2) = __float2bfloat16(pv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (threadIdx.x == 0) MTC_TRACE(3, i);
      mbar_arrive(&pready[s]);
    }
    if (ok && nb > 0)
      ok = softmax_bar_and(
          mbar_wait(&odone[(nb - 1) & 1], ((nb - 1) >> 1) & 1, s_err, p.err, kErrWaitTimeoutEpilogue));
    if (ok) {
      // sums over the 64 token rows: lanes, then the 4 warps
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float v = l_part[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        l_part[h] = v;
      }
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < HG; h += 4)
          *reinterpret_cast<float4*>(sLsum + warp * HG + h) = make_float4(l_part[h], l_part[h + 1], l_part[h + 2], l_part[h + 3]);
      }
      softmax_bar();
      float inv[HG];
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        const float l = sLsum[h] + sLsum[HG + h] + sLsum[2 * HG + h] + sLsum[3 * HG + h];
        l_part[h] = l;
        inv[h] = l > 0.f ? 1.f / l : 0.f;
      }
      tc_fence_after();
      const int head0 = hg * HG;
      const long long prow = ((long long)b * p.splits + split) * p.H + head0;
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        float ov[HG];
        if (nb > 0) {
          tmem_ld_cols<HG>(t_lane + C::O_COL + k * HG, ov);
        } else {
#pragma unroll
          for (int h = 0; h < HG; ++h) ov[h] = 0.f;
        }
        const int d = k * 128 + warp * 32 + lane;
        if (p.splits == 1) {
#pragma unroll
          for (int h = 0; h < HG; ++h)
            p.out[((long long)b * p.H + head0 + h) * MLA_LAT + d] = __float2bfloat16(ov[h] * inv[h]);
        } else {
#pragma unroll
          for (int h = 0; h < HG; ++h) p.o_part[(prow + h) * MLA_LAT + d] = ov[h] * inv[h];
        }
      }
      if (p.splits > 1 && threadIdx.x < HG) {
        // one head per thread: its max and sum are the same in every softmax thread
        float mh = -INFINITY, lh = 0.f;
#pragma unroll
        for (int h = 0; h < HG; ++h)
          if (h == (int)threadIdx.x) { mh = m_run[h]; lh = l_part[h]; }
        p.lse_part[prow + threadIdx.x] = lh > 0.f ? mh + __log2f(lh) : -INFINITY;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) MTC_TRACE(5, 1);
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc<C::TMEM_COLS>(tbase);
  }
}
#undef MTC_TRACE

template <int HG>
static void launch_mla_tc(const MlaDecodeLaunch& l) {
  using C = MtcCfg<HG>;
  CUtensorMap tq, tkv;
  make_tmap_2d(&tq, l.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (long long)l.B * l.H, MLA_DIM, MLA_DIM, HG, 64);
  make_tmap_2d(&tkv, l.cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.num_slots, MLA_DIM, MLA_DIM, mtc::TOK, 64);
  auto kern = mla_decode_tc_kernel<HG>;
  set_smem_bytes(kern, C::SMEM);
  MlaKParams p;
  p.block_table = l.block_table;
  p.max_blocks = l.max_blocks;
  p.context_lens = l.context_lens;
  p.out = (bf16*)l.out;
  p.o_part = l.o_part;
  p.lse_part = l.lse_part;
  p.B = l.B;
  p.H = l.H;
  p.splits = l.splits;
  p.scale_log2 = l.scale * 1.4426950408889634f;
  p.err = l.err;
  p.trace = l.trace;
  p.last_slot = nullptr;
  p.cache = (const bf16*)l.cache;
  if (l.B > 65535 || l.splits > 65535) throw std::runtime_error("mla_decode: batch / splits beyond the grid limits");
  launch_k(kern, dim3(l.H / HG, l.B, l.splits), dim3(C::THREADS), C::SMEM, l.stream, tq, tkv, p);
  if (l.splits > 1) {
    launch_k(mla_combine_kernel, dim3(l.B * l.H), dim3(MLA_LAT / 4), 0, l.stream, (const float*)l.o_part,
             (const float*)l.lse_part, (bf16*)l.out, l.H, l.splits);
  }
}

template <int HG, int NJ, int TOK, bool SPLIT = false, int NST = 2>
static void launch_mla(const MlaDecodeLaunch& l) {
  using C = MlaCfg<HG, NJ, TOK, NST>;
  CUtensorMap tq, tkv;
  make_tmap_2d(&tq, l.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (long long)l.B * l.H, MLA_DIM, MLA_DIM, HG, 64);
  make_tmap_2d(&tkv, l.cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, l.num_slots, MLA_DIM, MLA_DIM, TOK, 64);
  auto kern = l.last_slot ? mla_decode_kernel<HG, NJ, TOK, true, SPLIT, NST>
                          : mla_decode_kernel<HG, NJ, TOK, false, SPLIT, NST>;
  set_smem_bytes(kern, C::SMEM);
  MlaKParams p;
  p.block_table = l.block_table;
  p.max_blocks = l.max_blocks;
  p.context_lens = l.context_lens;
  p.out = (bf16*)l.out;
  p.o_part = l.o_part;
  p.lse_part = l.lse_part;
  p.B = l.B;
  p.H = l.H;
  p.splits = l.splits;
  p.scale_log2 = l.scale * 1.4426950408889634f;
  p.err = l.err;
  p.trace = nullptr;
  p.last_slot = l.last_slot;
  p.cache = (const bf16*)l.cache;
  if (l.B > 65535 || l.splits > 65535) throw std::runtime_error("mla_decode: batch / splits beyond the grid limits");
  dim3 grid(l.H / HG, l.B, l.splits);
  launch_k(kern, grid, dim3(C::WARPS * 32), C::SMEM, l.stream, tq, tkv, p);
  if (l.splits > 1) {
    launch_k(mla_combine_kernel, dim3(l.B * l.H), dim3(MLA_LAT / 4), 0, l.stream, (const float*)l.o_part,
             (const float*)l.lse_part, (bf16*)l.out, l.H, l.splits);
  }
}

// Tokens per KV stage of the mma.sync kernel: 64 (default) or 32
// (SPARKPIPE_MLA_STAGE_TOKENS=32). Measured with utils/bench_attention.py at the best
// split each: B=64, 16 heads, ctx 1024: 25.4 us (64) vs 27.8 us (32); B=32, 64 heads,
// ctx 2048: 57.5 us vs 66.6 us. Twice the CTAs per SM did not pay for twice the
// per-stage synchronisation.
int mla_stage_tokens() {
  static const int t = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_STAGE_TOKENS");
    return (e && std::string(e) == "32") ? 32 : 64;
  }();
  return t;
}

// Default decode kernel: the mma.sync one; SPARKPIPE_MLA_KERNEL=tc selects the
// tcgen05 kernel. Measured with utils/bench_attention.py (CUDA-graph replays):
// B=64, 16 heads, ctx 1024: 25.2 us (mma.sync) vs 34.2 us (tcgen05); B=32, 64 heads,
// ctx 2048: 57.1 us vs 58.7 us. A device trace of one tcgen05 CTA (the `trace`
// argument) shows why: each tcgen05.mma of these shapes (M=64 or 128, N = 16-32
// heads, K=16) occupies the tensor pipe ~45 ns whatever its size, so the 52
// instructions of a 64-token tile take ~2.3 us; with 72 KB stages only two fit
// beside Q, and the stream stalls behind the tensor pipe. Wider N (all 64 heads of
// a 64-head model in one CTA) does not fit shared memory with double buffering.
int mla_default_impl() {
  static const int t = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_KERNEL");
    return (e && std::string(e) == "tc") ? MLA_IMPL_TC : MLA_IMPL_MMA;
  }();
  return t;
}

// Warp layout of the 16-head, 64-token mma.sync kernel: SPARKPIPE_MLA_WARPS=8 splits
// each stage's tokens and latent columns over 8 warps instead of 4 (measured slower:
// 27.1 vs 25.0 us at B=64, 16 heads, ctx 1024). The S product's two accumulator
// chains are the default (25.0 vs 25.3 us there, 56.9 vs 57.2 us at B=32, 64 heads,
// ctx 2048); SPARKPIPE_MLA_SPLIT_ACC=0 uses one chain.
int mla_warps16() {
  static const int w = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_WARPS");
    return (e && std::string(e) == "8") ? 8 : 4;
  }();
  return w;
}
// KV stages in flight (SPARKPIPE_MLA_STAGES): 2 by default. With 32-token stages, 4
// keeps four in flight (the shared memory of two 64-token ones): measured slower, 33.1
// vs 25.2 us (B=64, 16 heads, ctx 1024, best split each), so the stage pipeline is not
// starved by load latency. With 64-token stages and 16 heads, 1 leaves each CTA one
// stage buffer and fits two CTAs per SM, each SM sub-partition then running two warps
// whose loads and math interleave.
int mla_stages() {
  static const int v = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_STAGES");
    if (e && std::string(e) == "4") return 4;
    if (e && std::string(e) == "1") return 1;
    return 2;
  }();
  return v;
}
int mla_stages32() { return mla_stages() == 4 ? 4 : 2; }
bool mla_single_stage16() { return mla_stages() == 1; }
bool mla_split_acc() {
  static const bool v = [] {
    const char* e = std::getenv("SPARKPIPE_MLA_SPLIT_ACC");
    return !(e && std::string(e) == "0");
  }();
  return v;
}

int mla_ctas_per_sm(int heads, int impl) {
  if (impl == MLA_IMPL_AUTO) impl = mla_default_impl();
  if (impl == MLA_IMPL_TC) return 1;
  const int tok = mla_stage_tokens();
  const bool deep = mla_stages32() == 4;
  if (heads % 32 == 0) {
    if (tok == 64) return MlaCfg<32, 4, 64>::MIN_CTAS;
    return deep ? MlaCfg<32, 4, 32, 4>::MIN_CTAS : MlaCfg<32, 4, 32>::MIN_CTAS;
  }
  if (tok == 64 && mla_warps16() == 8) return MlaCfg<16, 8, 64>::MIN_CTAS;
  if (tok == 64 && mla_single_stage16()) return MlaCfg<16, 4, 64, 1>::MIN_CTAS;
  if (tok == 64) return MlaCfg<16, 4, 64>::MIN_CTAS;
  return deep ? MlaCfg<16, 4, 32, 4>::MIN_CTAS : MlaCfg<16, 4, 32>::MIN_CTAS;
}

void mla_decode(const MlaDecodeLaunch& l) {
  if (l.B <= 0) return;
  if (l.kv_lora != MLA_LAT || l.rope != 64 || l.block_size != MLA_BLK)
    throw std::runtime_error("mla_decode: supports kv_lora 512, rope 64, 64-token blocks");
  if (l.splits > 1 && (!l.o_part || !l.lse_part)) throw std::runtime_error("mla_decode: split-KV needs scratch");
  if (l.H % 16 != 0) throw std::runtime_error("mla_decode: heads must be a multiple of 16");
  const int impl = l.impl == MLA_IMPL_AUTO ? mla_default_impl() : l.impl;
  if (impl == MLA_IMPL_TC && l.last_slot) throw std::runtime_error("mla_decode: last_slot needs the mma.sync kernel");
  if (impl == MLA_IMPL_TC) {
    if (l.H % 32 == 0) launch_mla_tc<32>(l);
    else launch_mla_tc<16>(l);
    return;
  }
  if (l.H % 32 == 0) {
    if (mla_stage_tokens() == 64) {
      if (mla_split_acc()) launch_mla<32, 4, 64, true>(l);
      else launch_mla<32, 4, 64>(l);
    } else if (mla_stages32() == 4) {
      launch_mla<32, 4, 32, true, 4>(l);
    } else {
      launch_mla<32, 4, 32>(l);
    }
  } else if (mla_stage_tokens() == 64) {
    const bool sp = mla_split_acc();
    if (mla_warps16() == 8) {
      if (sp) launch_mla<16, 8, 64, true>(l);
      else launch_mla<16, 8, 64>(l);
    } else if (mla_single_stage16()) {
      launch_mla<16, 4, 64, true, 1>(l);
    } else {
      if (sp) launch_mla<16, 4, 64, true>(l);
      else launch_mla<16, 4, 64>(l);
    }
  } else if (mla_stages32() == 4) {
    launch_mla<16, 4, 32, true, 4>(l);
  } else {
    launch_mla<16, 4, 32>(l);
  }
}

void kernel_attrs_mla(std::vector<KernelAttr>& out) {
  push_kernel_attr(out, "mla_decode_kernel<16,4,64>", mla_decode_kernel<16, 4, 64>);
  push_kernel_attr(out, "mla_decode_kernel<32,4,64>", mla_decode_kernel<32, 4, 64>);
  push_kernel_attr(out, "mla_decode_tc_kernel<16>", mla_decode_tc_kernel<16>);
  push_kernel_attr(out, "mla_decode_tc_kernel<32>", mla_decode_tc_kernel<32>);
  push_kernel_attr(out, "mla_combine_kernel", mla_combine_kernel);
}

}  // namespace sp
