// Chunked / paged prefill attention for MLA in its expanded (non-absorbed) form:
//
//   q = [q_nope (dn) | q_pe (dr)],  k = [k_nope (dn) | k_pe (dr, shared by heads)],  v (dv)
//   o[i] = softmax_j<=limit(i) (scale * q[i] . k[j]) v[j]
//
// Variable-length batches via cu_q / cu_k prefix arrays. The key range of a
// sequence may be longer than its query chunk (cached prefix + chunk): query i of
// a chunk of length Lq against Lk keys sees keys j <= Lk - Lq + i.
//
// Flash-attention style: one CTA = 64 queries of one head, 4 warps x 16 rows,
// 64-key tiles double buffered with cp.async into 128-byte-swizzled shared
// tiles, online softmax in registers, P reused as the A operand of P.V.
//
// Reference: PagedPrefillPlan / BulkPrefillPlan in
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:736-779.
#include <cuda_runtime.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"
#include "mma_sync.cuh"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {
constexpr int QT = 64;   // queries per CTA
constexpr int KT = 64;   // keys per tile
constexpr int DN = 128, DR = 64, DQK = 192, DV = 128;
constexpr int SUB = KT * 128;  // one [64 x 64] bf16 swizzled sub-tile
constexpr int OFF_Q = 0;                       // 3 sub-tiles
constexpr int OFF_K = 3 * SUB;                 // 2 x 3 sub-tiles
constexpr int OFF_V = OFF_K + 2 * 3 * SUB;     // 2 x 2 sub-tiles
constexpr int SMEM = OFF_V + 2 * 2 * SUB + 1024;

SP_DEVI void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
SP_DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SP_DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
SP_DEVI uint32_t chunk_addr(uint32_t base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}
}  // namespace

__global__ void __launch_bounds__(128, 2) prefill_attn_kernel(const PrefillAttnLaunch p, float scale_log2) {
  griddep_wait();
  griddep_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const int b = blockIdx.z, h = blockIdx.y;
  const int q_begin = p.cu_q[b], q_len = p.cu_q[b + 1] - q_begin;
  const int k_begin = p.cu_k[b], k_len = p.cu_k[b + 1] - k_begin;
  const int q0 = blockIdx.x * QT;
  if (q0 >= q_len) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int diag = k_len - q_len;  // query i sees keys <= diag + i
  int kend = p.causal ? min(k_len, diag + q0 + QT) : k_len;
  const int n_kt = kend > 0 ? (kend + KT - 1) / KT : 0;

  const bf16* Q = reinterpret_cast<const bf16*>(p.q);
  const bf16* K = reinterpret_cast<const bf16*>(p.k);
  const bf16* KPE = reinterpret_cast<const bf16*>(p.kpe);
  const bf16* V = reinterpret_cast<const bf16*>(p.v);

  // Q tile: 64 rows x 24 chunks
  for (int c = tid; c < QT * 24; c += 128) {
    const int r = c / 24, ch = c % 24;
    const int qi = q0 + r;
    const bool valid = qi < q_len;
    const bf16* src = Q + (long long)(q_begin + (valid ? qi : 0)) * p.q_tok + (long long)h * p.q_head + ch * 8;
    cp_async16(chunk_addr(s0 + OFF_Q + (ch >> 3) * SUB, r, ch & 7), src, valid);
  }
  auto load_kv = [&](int kt, int buf) {
    const uint32_t kb = s0 + OFF_K + buf * 3 * SUB;
    const uint32_t vb = s0 + OFF_V + buf * 2 * SUB;
    for (int c = tid; c < KT * 40; c += 128) {
      const int r = c / 40, ch = c % 40;
      const int kj = kt * KT + r;
      const bool valid = kj < k_len;
      const long long tok = k_begin + (valid ? kj : 0);
      if (ch < 16) {
        cp_async16(chunk_addr(kb + (ch >> 3) * SUB, r, ch & 7), K + tok * p.k_tok + (long long)h * p.k_head + ch * 8,
                   valid);
      } else if (ch < 24) {
        cp_async16(chunk_addr(kb + 2 * SUB, r, ch - 16), KPE + tok * p.kpe_tok + (ch - 16) * 8, valid);
      } else {
        const int vc = ch - 24;
        cp_async16(chunk_addr(vb + (vc >> 3) * SUB, r, vc & 7), V + tok * p.v_tok + (long long)h * p.v_head + vc * 8,
                   valid);
      }
    }
  };
  if (n_kt > 0) load_kv(0, 0);
  cp_commit();

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int r_lo = lane >> 2;
  const int row_q0 = q0 + warp * 16 + r_lo;  // query index (within the chunk) of fragment row r_lo

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) load_kv(kt + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t kb = s0 + OFF_K + buf * 3 * SUB;
    const uint32_t vb = s0 + OFF_V + buf * 2 * SUB;

    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DQK / 16; ++kk) {
      const int sub = kk >> 2, cc = (kk & 3) * 16;
      uint32_t a[4];
      ldsm_x4(a, swz128(s0 + OFF_Q + sub * SUB, warp * 16 + (lane & 15), cc + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        ldsm_x4(bb, swz128(kb + sub * SUB, np * 16 + (lane & 7) + (lane >> 4) * 8, cc + ((lane >> 3) & 1) * 8));
        mma16816(sc[2 * np], a, bb[0], bb[1]);
        mma16816(sc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = kt * KT + n * 8 + (lane & 3) * 2 + (e & 1);
        const int qi = row_q0 + (e >> 1) * 8;
        float v = sc[n][e] * scale_log2;
        if (kj >= k_len || (p.causal && kj > diag + qi)) v = -INFINITY;
        sc[n][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
      const float mn = fmaxf(m_run[hh], mx[hh]);
      alpha[hh] = (m_run[hh] == -INFINITY) ? 0.f : exp2f(m_run[hh] - mn);
      m_run[hh] = mn;
      l_run[hh] *= alpha[hh];
    }
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mrow = m_run[e >> 1];
        pv[e] = (sc[n][e] == -INFINITY || mrow == -INFINITY) ? 0.f : exp2f(sc[n][e] - mrow);
        l_run[e >> 1] += pv[e];
      }
      pa[n >> 1][(n & 1) * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
      o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      // A fragment order: (rows lo, k lo), (rows hi, k lo), (rows lo, k hi), (rows hi, k hi)
      uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
      const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        const int dim = np * 16 + (lane >> 4) * 8;
        uint32_t bb[4];
        ldsm_x4_t(bb, swz128(vb + (dim >> 6) * SUB, tok, dim & 63));
        mma16816(o[2 * np], a, bb[0], bb[1]);
        mma16816(o[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 1);
    l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 2);
  }
  bf16* O = reinterpret_cast<bf16*>(p.o);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int qi = row_q0 + hh * 8;
    if (qi >= q_len) continue;
    const float inv = l_run[hh] > 0.f ? 1.f / l_run[hh] : 0.f;
    bf16* orow = O + (long long)(q_begin + qi) * p.o_tok + (long long)h * p.o_head + (lane & 3) * 2;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(orow + n * 8) = pack_bf16(o[n][2 * hh] * inv, o[n][2 * hh + 1] * inv);
  }
}

// Default: the tcgen05 kernel (prefill_attn_tc.cu) when the tensors suit TMA;
// SPARKPIPE_ATTN_KERNEL=mma selects this mma.sync kernel.
static int attn_default_impl() {
  static const int t = [] {
    const char* e = std::getenv("SPARKPIPE_ATTN_KERNEL");
    return (e && std::string(e) == "mma") ? ATTN_IMPL_MMA : ATTN_IMPL_TC;
  }();
  return t;
}

void prefill_attention(const PrefillAttnLaunch& l) {
  if (l.B <= 0 || l.max_q <= 0) return;
  if (l.dn != DN || l.dr != DR || l.dv != DV)
    throw std::runtime_error("prefill_attention: supports dn 128, dr 64, dv 128");
  const int impl = l.impl == ATTN_IMPL_AUTO ? attn_default_impl() : l.impl;
  if (impl == ATTN_IMPL_TC && prefill_attention_tc_ok(l)) {
    prefill_attention_tc(l);
    return;
  }
  set_smem_bytes(prefill_attn_kernel, SMEM);
  dim3 grid((l.max_q + QT - 1) / QT, l.H, l.B);
  launch_k(prefill_attn_kernel, grid, dim3(128), SMEM, l.stream, l, l.scale * 1.4426950408889634f);
}

}  // namespace sp
