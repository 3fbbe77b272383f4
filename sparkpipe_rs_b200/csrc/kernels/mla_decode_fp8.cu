// MLA paged decode attention over an fp8 (e4m3) latent KV cache, sm_100a.
//
// Cache format (one layer):
//   cache8 [slots, 576] e4m3: the token's [latent (512) | rope key (64)] row;
//   scales [slots, 5] fp32:    value = e4m3 * scale, one scale per 128-element block of
//                              the row (blocks 0-3: latent, block 4: the 64 rope dims),
//                              scale = amax(block) / 448 chosen when the token is written.
// A row is 576 + 20 bytes against 1,152 in bf16 (0.52x of the bytes a decode step
// streams; twice the tokens per GB of HBM).
//
// Same decomposition as the bf16 mma.sync kernel (mla_decode.cu): one CTA per (head
// group, sequence, KV split), 64-token stages streamed by TMA (nine 64-byte-wide boxes,
// 64-byte swizzle) plus one bulk copy of the stage's 64 x 5 scales, four warps per
// 16-head tile, split-KV partials merged by the shared combine kernel. The products
// run on mma.sync m16n8k16 with f16 operands: e4m3 converts exactly to f16 two values
// per instruction, and the fp8 bytes are read straight from the stage:
//
//   S = Q K^T: ldmatrix (non-transposed, 16-bit units) hands each thread four
//     consecutive fp8 dims 4t..4t+3 of one token; the MMA reads them as the k indices
//     (2t, 2t+1, 2t+8, 2t+9). Q is converted once per CTA to f16 with the same
//     permutation inside every 16-dim group, so sum_k Q[k] K[k] is unchanged. Partial
//     sums of each 128-dim block are scaled by the token's block scale.
//   O = P V: ldmatrix.trans on the fp8 stage gives each thread the byte pairs of two
//     consecutive tokens at dims (2g, 2g+1); one byte permute splits them into the
//     token pairs of dim 2g and of dim 2g+1, so each 16-dim group feeds two n8 tiles
//     (even and odd dims). The V scales (token x 128-dim block) fold into P: warp j
//     owns latent block j, multiplies its P fragments by scale[t][j] / f_j (f_j the
//     stage's largest block-j scale, so the f16 factors stay in [0, 1]) and keeps its
//     accumulator in units of f_j, re-based with the softmax correction each stage.
//
// Reference: the fp8 KV cache plan with dynamic per-128 scales,
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:47-56, 624-644.
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "mma_sync.cuh"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {

constexpr int K8_DIM = 576;
constexpr int K8_LAT = 512;
constexpr int K8_NSCALE = 5;
constexpr int K8_CHUNKS = 9;   // 64-dim boxes per row
constexpr int K8_TOK = 64;     // tokens per stage = one cache block

template <int HG, int NST>
struct Mla8Cfg {
  static constexpr int NJ = 4;
  static constexpr int WARPS = NJ * (HG / 16);
  static constexpr int CHUNK_BYTES = K8_TOK * 64;             // one 64-token x 64-dim fp8 box
  static constexpr int KV_BYTES = K8_CHUNKS * CHUNK_BYTES;      // 36,864
  static constexpr int SCL_BYTES = K8_TOK * K8_NSCALE * 4;      // 1,280
  static constexpr int Q_BYTES = K8_CHUNKS * HG * 128;          // bf16 Q, later f16 in place
  static constexpr int P_PITCH = K8_TOK + 8;                    // f16 elements per P row
  static constexpr int OFF_KV = (Q_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_SCL = OFF_KV + NST * KV_BYTES;
  static constexpr int OFF_P = OFF_SCL + NST * SCL_BYTES;
  static constexpr int OFF_STAT = OFF_P + HG * P_PITCH * 2;
  static constexpr int OFF_BAR = OFF_STAT + 2 * NJ * HG * 4;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;
  static constexpr int MIN_CTAS = (2 * (SMEM + 1024) <= 228 * 1024) ? 2 : 1;
};

struct Mla8Params {
  const int* block_table;
  int max_blocks;
  const int* context_lens;
  const float* scales;      // [slots, 5]
  const uint8_t* cache8;    // [slots, 576]
  bf16* out;
  float* o_part;
  float* lse_part;
  int B, H, splits;
  float scale_log2;
  int* err;
  const int* last_slot;
};

SP_DEVI void mma16816_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two e4m3 values (low byte first) -> f16x2 (exact)
SP_DEVI uint32_t e4m3x2_f16x2(uint32_t v16) {
  uint32_t r;
  const unsigned short h = (unsigned short)(v16 & 0xffffu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}

SP_DEVI uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 x = *reinterpret_cast<__half2*>(&a), y = *reinterpret_cast<__half2*>(&b);
  __half2 z = __hmul2(x, y);
  return *reinterpret_cast<uint32_t*>(&z);
}

SP_DEVI uint32_t pack_f16(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// byte offset of (token, 16-byte unit u) in a 64-token x 64-byte box written with the 64-byte swizzle
SP_DEVI uint32_t swz64(int token, int u) { return token * 64 + ((u ^ ((token >> 1) & 3)) << 4); }

template <int HG, int NST, bool LAST>
__global__ void __launch_bounds__(Mla8Cfg<HG, NST>::WARPS * 32, Mla8Cfg<HG, NST>::MIN_CTAS)
    mla_decode_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                          const Mla8Params p) {
  griddep_wait();
  griddep_launch();
  using C = Mla8Cfg<HG, NST>;
  constexpr int NJ = C::NJ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = smem_u32(smem + C::OFF_KV);
  float* sScl = reinterpret_cast<float*>(smem + C::OFF_SCL);
  __half* sP = reinterpret_cast<__half*>(smem + C::OFF_P);
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
  const int nblk = (ctx + K8_TOK - 1) / K8_TOK;
  const int per = (nblk + p.splits - 1) / p.splits;
  const int kb0 = min(nblk, split * per);
  const int kb1 = min(nblk, kb0 + per);
  const int nb = max(0, kb1 - kb0);
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

  auto issue_block = [&](int i) {  // thread 0 only
    const int s = i % NST;
    const int row = bt[kb0 + i] * K8_TOK;
    uint64_t* bar = &full[s];
    mbar_arrive_expect_tx(bar, C::KV_BYTES + C::SCL_BYTES);
    uint8_t* dst = smem + C::OFF_KV + s * C::KV_BYTES;
#pragma unroll 1
    for (int c = 0; c < K8_CHUNKS; ++c) tma_load_2d(dst + c * C::CHUNK_BYTES, &tmKV, bar, c * 64, row);
    bulk_load(sScl + s * K8_TOK * K8_NSCALE, p.scales + (long long)row * K8_NSCALE, C::SCL_BYTES, bar);
  };
  int issued = 0;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(qbar, C::Q_BYTES);
    for (int c = 0; c < K8_CHUNKS; ++c) tma_load_2d(smem + c * HG * 128, &tmQ, qbar, c * 64, b * p.H + hg * HG);
    for (; issued < NST && issued < nb; ++issued) issue_block(issued);
  }

  bool ok = mbar_wait(qbar, 0, s_err, p.err, kErrWaitTimeoutMma);
  ok = __syncthreads_and(ok);
  if (ok) {
    // Q: bf16 -> f16, each 16-dim group permuted so that logical k (2t, 2t+1, 2t+8, 2t+9)
    // holds dims (4t .. 4t+3): new[0..7] = old[0,1,4,5,8,9,12,13], new[8..15] = old[2,3,6,7,...].
    for (int w = threadIdx.x; w < HG * 36; w += blockDim.x) {
      const int row = w / 36, g16 = w % 36;
      const int c = g16 >> 2, u0 = (g16 & 3) * 2;
      uint8_t* base = smem + c * HG * 128 + row * 128;
      uint4* pa = reinterpret_cast<uint4*>(base + (((u0) ^ (row & 7)) << 4));
      uint4* pb = reinterpret_cast<uint4*>(base + (((u0 + 1) ^ (row & 7)) << 4));
      const uint4 va = *pa, vb = *pb;
      const uint32_t in[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};  // bf16 pairs (0,1) (2,3) ...
      uint32_t f[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&in[k]));
        f[k] = pack_f16(x.x, x.y);
      }
      // pairs: f[k] = dims (2k, 2k+1); new unit A = pairs 0,2,4,6; unit B = pairs 1,3,5,7
      *pa = make_uint4(f[0], f[2], f[4], f[6]);
      *pb = make_uint4(f[1], f[3], f[5], f[7]);
    }
    __syncthreads();
  }

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  float f_prev = 1.f;                   // accumulator unit of this warp's latent block
  const int r_lo = lane >> 2, tq = lane & 3;
  const int qrow = mt * 16;

  for (int i = 0; ok && i < nb; ++i) {
    const int s = i % NST;
    bool got = mbar_wait(&full[s], (i / NST) & 1, s_err, p.err, kErrWaitTimeoutMma);
    if (!__syncthreads_and(got)) { ok = false; break; }
    const uint32_t kvb = sKV + s * C::KV_BYTES;
    float* scl = sScl + s * K8_TOK * K8_NSCALE;
    if constexpr (LAST) {
      const int t_last = ctx - 1, t0 = (kb0 + i) * K8_TOK;
      const int src = p.last_slot[b];
      if (t_last >= t0 && t_last < t0 + K8_TOK && src >= 0 && src != bt[t_last / K8_TOK] * K8_TOK + t_last % K8_TOK) {
        const int tr = t_last - t0;
        uint8_t* st = smem + C::OFF_KV + s * C::KV_BYTES;
        for (int e = threadIdx.x; e < K8_CHUNKS * 4 + K8_NSCALE; e += blockDim.x) {
          if (e < K8_CHUNKS * 4) {
            const int c = e >> 2, u = e & 3;
            const uint4 v = *reinterpret_cast<const uint4*>(p.cache8 + (long long)src * K8_DIM + c * 64 + u * 16);
            *reinterpret_cast<uint4*>(st + c * C::CHUNK_BYTES + swz64(tr, u)) = v;
          } else {
            const int k = e - K8_CHUNKS * 4;
            scl[tr * K8_NSCALE + k] = p.scales[(long long)src * K8_NSCALE + k];
          }
        }
        fence_proxy_async_smem();
        __syncthreads();
      }
    }

    // ---- S = Q K^T: 16 heads x 16 tokens (two n8 tiles) per warp, per-128-dim block scaled
    float sc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int blk = 0; blk < K8_NSCALE; ++blk) {
      float ta[2][4], tb[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        ta[n][0] = ta[n][1] = ta[n][2] = ta[n][3] = 0.f;
        tb[n][0] = tb[n][1] = tb[n][2] = tb[n][3] = 0.f;
      }
      constexpr int PAIRS_FULL = 4;
      const int pairs = blk < 4 ? PAIRS_FULL : 2;
#pragma unroll
      for (int kp = 0; kp < PAIRS_FULL; ++kp) {
        if (kp < pairs) {
          const int kk0 = blk * 8 + kp * 2;           // first of two k16 steps (same 64-dim chunk)
          const int c = kk0 >> 2, u0 = kk0 & 3;
          uint32_t a0[4], a1[4], kb[4];
          ldsm_x4(a0, swz128(sQ + c * HG * 128, qrow + (lane & 15), u0 * 16 + (lane >> 4) * 8));
          ldsm_x4(a1, swz128(sQ + c * HG * 128, qrow + (lane & 15), (u0 + 1) * 16 + (lane >> 4) * 8));
          {
            const int m = lane >> 3;
            const int tok = j * 16 + (m & 1) * 8 + (lane & 7);
            ldsm_x4(kb, kvb + c * C::CHUNK_BYTES + swz64(tok, u0 + (m >> 1)));
          }
          mma16816_f16(ta[0], a0, e4m3x2_f16x2(kb[0]), e4m3x2_f16x2(kb[0] >> 16));
          mma16816_f16(ta[1], a0, e4m3x2_f16x2(kb[1]), e4m3x2_f16x2(kb[1] >> 16));
          mma16816_f16(tb[0], a1, e4m3x2_f16x2(kb[2]), e4m3x2_f16x2(kb[2] >> 16));
          mma16816_f16(tb[1], a1, e4m3x2_f16x2(kb[3]), e4m3x2_f16x2(kb[3] >> 16));
        }
      }
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int tk = j * 16 + n * 8 + tq * 2;
        const float s0 = scl[tk * K8_NSCALE + blk], s1 = scl[(tk + 1) * K8_NSCALE + blk];
        sc[n][0] += (ta[n][0] + tb[n][0]) * s0;
        sc[n][1] += (ta[n][1] + tb[n][1]) * s1;
        sc[n][2] += (ta[n][2] + tb[n][2]) * s0;
        sc[n][3] += (ta[n][3] + tb[n][3]) * s1;
      }
    }
    // ---- scale, mask, row max across the NJ warps of the head tile
    const int tok0 = (kb0 + i) * K8_TOK + j * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tok0 + n * 8 + tq * 2 + (e & 1);
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
    if (tq == 0) {
      sMax[j * HG + qrow + r_lo] = mx[0];
      sMax[j * HG + qrow + r_lo + 8] = mx[1];
    }
    // this warp's V block scale factors: f = max over the stage's tokens of scale[t][j]
    // (tokens past the context hold stale rows: they take no part)
    const int stage0 = (kb0 + i) * K8_TOK;
    const int nvalid = ctx - stage0;  // tokens of this stage inside the context (>= 1)
    auto vscale = [&](int t) { return t < nvalid ? scl[t * K8_NSCALE + j] : 0.f; };
    float fj = fmaxf(vscale(lane), vscale(lane + 32));
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) fj = fmaxf(fj, __shfl_xor_sync(0xffffffffu, fj, d));
    const float f_cur = fj > 0.f ? fj : 1.f;
    const float inv_f = 1.f / f_cur;
    uint32_t rr[4][2];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int t0 = kk * 16 + tq * 2;
      rr[kk][0] = pack_f16(vscale(t0) * inv_f, vscale(t0 + 1) * inv_f);
      rr[kk][1] = pack_f16(vscale(t0 + 8) * inv_f, vscale(t0 + 9) * inv_f);
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
    // ---- P = exp2(S - m) as f16 (unscaled; each warp applies its V scales)
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[e] = (sc[n][e] == -INFINITY) ? 0.f : exp2f(sc[n][e] - m_run[e >> 1]);
        l_run[e >> 1] += pv[e];
      }
      const int col = j * 16 + n * 8 + tq * 2;
      *reinterpret_cast<uint32_t*>(sP + (qrow + r_lo) * C::P_PITCH + col) = pack_f16(pv[0], pv[1]);
      *reinterpret_cast<uint32_t*>(sP + (qrow + r_lo + 8) * C::P_PITCH + col) = pack_f16(pv[2], pv[3]);
    }
    const float rebase = f_prev * inv_f;
    f_prev = f_cur;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha[0] * rebase; o[n][1] *= alpha[0] * rebase;
      o[n][2] *= alpha[1] * rebase; o[n][3] *= alpha[1] * rebase;
    }
    __syncthreads();
    // ---- O[16 heads, 128 dims of block j] += (P * scale[:, j] / f) V
    const uint32_t sPa = smem_u32(sP);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sPa + ((qrow + (lane & 15)) * C::P_PITCH + kk * 16 + (lane >> 4) * 8) * 2);
      a[0] = hmul2_u32(a[0], rr[kk][0]);
      a[1] = hmul2_u32(a[1], rr[kk][0]);
      a[2] = hmul2_u32(a[2], rr[kk][1]);
      a[3] = hmul2_u32(a[3], rr[kk][1]);
      const int m = lane >> 3;
      const int tok = kk * 16 + (m & 1) * 8 + (lane & 7);
#pragma unroll
      for (int gp = 0; gp < 4; ++gp) {
        const int G = j * 8 + gp * 2 + (m >> 1);     // 16-dim group of this lane's matrix row
        uint32_t v[4];
        ldsm_x4_t(v, kvb + (G >> 2) * C::CHUNK_BYTES + swz64(tok, G & 3));
        const uint32_t p0 = __byte_perm(v[0], 0, 0x3120), p1 = __byte_perm(v[1], 0, 0x3120);
        const uint32_t p2 = __byte_perm(v[2], 0, 0x3120), p3 = __byte_perm(v[3], 0, 0x3120);
        mma16816_f16(o[gp * 4 + 0], a, e4m3x2_f16x2(p0), e4m3x2_f16x2(p1));
        mma16816_f16(o[gp * 4 + 1], a, e4m3x2_f16x2(p0 >> 16), e4m3x2_f16x2(p1 >> 16));
        mma16816_f16(o[gp * 4 + 2], a, e4m3x2_f16x2(p2), e4m3x2_f16x2(p3));
        mma16816_f16(o[gp * 4 + 3], a, e4m3x2_f16x2(p2 >> 16), e4m3x2_f16x2(p3 >> 16));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && issued < nb) { issue_block(issued); ++issued; }
  }

  if (!ok) {
    if (threadIdx.x == 0)
      for (int i2 = max(0, issued - NST); i2 < issued; ++i2) mbar_drain(&full[i2 % NST], (i2 / NST) & 1);
    return;
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  if (tq == 0) {
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
    inv[h] = l > 0.f ? f_prev / l : 0.f;
    lse[h] = l > 0.f ? m_run[h] + __log2f(l) : -INFINITY;
  }
  // tile (gp, q, par) holds, for row r and accumulator columns (2t, 2t+1), dims
  // G * 16 + 4t + par and G * 16 + 4t + 2 + par with G = j * 8 + gp * 2 + q
  const int head0 = hg * HG + qrow + r_lo;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const long long rowi = p.splits == 1 ? ((long long)b * p.H + head0 + h * 8)
                                         : (((long long)b * p.splits + split) * p.H + head0 + h * 8);
#pragma unroll
    for (int gp = 0; gp < 4; ++gp)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int d0 = (j * 8 + gp * 2 + q) * 16 + tq * 4;
        const float* ev = o[gp * 4 + q * 2];
        const float* od = o[gp * 4 + q * 2 + 1];
        const float x0 = ev[2 * h] * inv[h], x1 = od[2 * h] * inv[h];
        const float x2 = ev[2 * h + 1] * inv[h], x3 = od[2 * h + 1] * inv[h];
        if (p.splits == 1) {
          *reinterpret_cast<uint2*>(p.out + rowi * K8_LAT + d0) = make_uint2(pack_bf16(x0, x1), pack_bf16(x2, x3));
        } else {
          *reinterpret_cast<float4*>(p.o_part + rowi * K8_LAT + d0) = make_float4(x0, x1, x2, x3);
        }
      }
    if (p.splits > 1 && j == 0 && tq == 0) p.lse_part[rowi] = lse[h];
  }
}

void make_tmap_fp8_rows(CUtensorMap* map, const void* ptr, long long rows) {
  make_tmap_2d_swizzle(map, ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, K8_DIM, K8_DIM, K8_TOK, 64,
                       CU_TENSOR_MAP_SWIZZLE_64B);
}

template <int HG, int NST>
void launch_mla8(const MlaDecodeLaunch& l) {
  using C = Mla8Cfg<HG, NST>;
  CUtensorMap tq, tkv;
  make_tmap_2d(&tq, l.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (long long)l.B * l.H, K8_DIM, K8_DIM, HG, 64);
  make_tmap_fp8_rows(&tkv, l.cache, l.num_slots);
  auto kern = l.last_slot ? mla_decode_fp8_kernel<HG, NST, true> : mla_decode_fp8_kernel<HG, NST, false>;
  set_smem_bytes(kern, C::SMEM);
  Mla8Params p;
  p.block_table = l.block_table;
  p.max_blocks = l.max_blocks;
  p.context_lens = l.context_lens;
  p.scales = l.kv_scales;
  p.cache8 = (const uint8_t*)l.cache;
  p.out = (bf16*)l.out;
  p.o_part = l.o_part;
  p.lse_part = l.lse_part;
  p.B = l.B;
  p.H = l.H;
  p.splits = l.splits;
  p.scale_log2 = l.scale * 1.4426950408889634f;
  p.err = l.err;
  p.last_slot = l.last_slot;
  if (l.B > 65535 || l.splits > 65535) throw std::runtime_error("mla_decode_fp8: batch / splits beyond the grid limits");
  launch_k(kern, dim3(l.H / HG, l.B, l.splits), dim3(C::WARPS * 32), C::SMEM, l.stream, tq, tkv, p);
  if (l.splits > 1) mla_combine(l.o_part, l.lse_part, l.out, l.B, l.H, l.splits, l.stream);
}

// Stages in flight: SPARKPIPE_MLA8_STAGES=4 (one CTA per SM) instead of 2 (two CTAs
// per SM at 16 heads); read at every launch.
int mla8_stages() {
  const char* e = std::getenv("SPARKPIPE_MLA8_STAGES");
  return (e && e[0] == '4') ? 4 : 2;
}

}  // namespace

int mla_fp8_ctas_per_sm(int heads) {
  const bool deep = mla8_stages() == 4;
  if (heads % 32 == 0) return deep ? Mla8Cfg<32, 4>::MIN_CTAS : Mla8Cfg<32, 2>::MIN_CTAS;
  return deep ? Mla8Cfg<16, 4>::MIN_CTAS : Mla8Cfg<16, 2>::MIN_CTAS;
}

void mla_decode_fp8(const MlaDecodeLaunch& l) {
  if (l.B <= 0) return;
  if (l.kv_lora != K8_LAT || l.rope != 64 || l.block_size != K8_TOK)
    throw std::runtime_error("mla_decode_fp8: supports kv_lora 512, rope 64, 64-token blocks");
  if (!l.kv_scales) throw std::runtime_error("mla_decode_fp8: the fp8 cache needs its scales");
  if ((reinterpret_cast<uintptr_t>(l.kv_scales) & 15) != 0)
    throw std::runtime_error("mla_decode_fp8: scales must be 16-byte aligned");
  if (l.splits > 1 && (!l.o_part || !l.lse_part)) throw std::runtime_error("mla_decode_fp8: split-KV needs scratch");
  if (l.H % 16 != 0) throw std::runtime_error("mla_decode_fp8: heads must be a multiple of 16");
  const bool deep = mla8_stages() == 4;
  if (l.H % 32 == 0) {
    if (deep) launch_mla8<32, 4>(l);
    else launch_mla8<32, 2>(l);
  } else {
    if (deep) launch_mla8<16, 4>(l);
    else launch_mla8<16, 2>(l);
  }
}

// ---------------------------------------------------------------- cache rows
// Dequantise cache rows: out[r, :] = cache8[idx[r], :] * scales[idx[r], block] (bf16).
__global__ void kv8_gather_kernel(const uint8_t* __restrict__ cache8, const float* __restrict__ scales,
                                  const int* __restrict__ idx, bf16* __restrict__ out, int n) {
  griddep_wait();
  griddep_launch();
  const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-byte unit per thread
  if (w >= (long long)n * (K8_DIM / 8)) return;
  const int r = (int)(w / (K8_DIM / 8)), u = (int)(w % (K8_DIM / 8));
  const long long src = idx[r];
  const float sc = scales[src * K8_NSCALE + (u * 8) / 128];
  const uint2 v = *reinterpret_cast<const uint2*>(cache8 + src * K8_DIM + u * 8);
  const uint32_t wv[2] = {v.x, v.y};
  uint32_t o4[4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t lo = e4m3x2_f16x2(wv[k]), hi = e4m3x2_f16x2(wv[k] >> 16);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    o4[2 * k] = pack_bf16(a.x * sc, a.y * sc);
    o4[2 * k + 1] = pack_bf16(c.x * sc, c.y * sc);
  }
  *reinterpret_cast<uint4*>(out + (long long)r * K8_DIM + u * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

void kv8_gather(const void* cache8, const float* scales, const int* idx, void* out, int n, cudaStream_t s) {
  if (n <= 0) return;
  const long long units = (long long)n * (K8_DIM / 8);
  launch_k(kv8_gather_kernel, dim3((unsigned)((units + 255) / 256)), dim3(256), 0, s, (const uint8_t*)cache8, scales,
           idx, (bf16*)out, n);
}

void kernel_attrs_mla8(std::vector<KernelAttr>& out) {
  push_kernel_attr(out, "mla_decode_fp8_kernel<16,2>", mla_decode_fp8_kernel<16, 2, false>);
  push_kernel_attr(out, "mla_decode_fp8_kernel<32,2>", mla_decode_fp8_kernel<32, 2, false>);
}

}  // namespace sp
