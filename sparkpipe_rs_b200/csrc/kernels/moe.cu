// Mixture-of-experts routing and token layout kernels, sm_100a.
//
//  * moe_topk     — router logits (from split-K slabs of the gate GEMM, or computed
//                   in the kernel from the token row and the gate for small routers),
//                   router scores (softmax, or sigmoid with a selection bias as in
//                   the noaux_tc routers), top-k selection, optional renormalisation
//                   and the routed scaling factor. Shared experts are appended as
//                   always-selected experts E .. E+S-1 with weight 1, so they run
//                   inside the same grouped GEMM as the routed experts.
//  * moe_align    — expert histogram -> per-expert row offsets and n-tile prefix
//                   counts (the device-side tile schedule of the grouped GEMM) ->
//                   scatter of (token, slot) pairs into expert-sorted rows. Decode
//                   sized problems run in one CTA (shared-memory histogram); large
//                   ones use grid-wide atomics in three kernels.
//  * gather_rows / silu_mul / moe_combine — row gather into the sorted layout,
//                   SwiGLU activation, and the top-k weighted scatter-add back.
//
// Reference: FAST_MOE_ROUTER fields (moe_router_weight_bf16, score bias, routed
// scaling factor, norm_topk_prob, topk ids/weights) of the resident decode stage
// node context, crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:869-1010,
// and the fused top-k reduce of the FP8 MoE entry point (:321-342, :1053).
#include <cuda_runtime.h>

#include <algorithm>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

constexpr int TOPK_MAX_PER_LANE = 16;  // E <= 512
constexpr int TOPK_THREADS = 256;
constexpr int TOPK_MAX_E = 32 * TOPK_MAX_PER_LANE;

// One CTA per token. The router logits arrive as `splits` fp32 split-K slabs: all
// 256 threads load them at once (thread = (slab group g, VEC-wide column chunk v),
// slabs g, g+G, ...), partial sums go through shared memory and are added in a
// fixed order, so the result does not depend on timing. Warp 0 then scores,
// optionally restricts the choice to the best `topk_group` of `n_group` expert
// groups (group score: the group's best expert, or the sum of its best two as in
// the bias-corrected sigmoid routers), and picks the top k by k rounds of a warp
// argmax (ties to the lower expert id).
// Scores one token's router logits (s_logit: E values in shared memory, read by
// lane e + 32 i), restricts to the best expert groups, picks the top k by k rounds
// of a warp argmax (ties to the lower expert id) and writes ids / weights (the
// shared experts follow as E, E + 1, ... with weight 1). One warp; s_scratch holds
// E floats for the group scores.
SP_DEVI void route_token_warp(const float* s_logit, float* s_scratch, int t, int lane, const float* __restrict__ bias,
                              int* __restrict__ ids, float* __restrict__ wts, int E, int k, int n_shared, int scoring,
                              int renorm, float scaling, int n_group, int topk_group, int group_top2) {
  float score[TOPK_MAX_PER_LANE], sel[TOPK_MAX_PER_LANE];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
    const int e = lane + i * 32;
    score[i] = (i < per && e < E) ? s_logit[e] : -INFINITY;
    mx = fmaxf(mx, score[i]);
  }
  if (scoring == 0) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      score[i] = (score[i] == -INFINITY) ? 0.f : __expf(score[i] - mx);
      sum += score[i];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      const int e = lane + i * 32;
      score[i] *= inv;
      sel[i] = (i < per && e < E) ? score[i] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      const int e = lane + i * 32;
      const bool valid = i < per && e < E;
      score[i] = valid ? 1.f / (1.f + __expf(-score[i])) : 0.f;
      sel[i] = valid ? score[i] + (bias ? bias[e] : 0.f) : -INFINITY;
    }
  }
  if (n_group > 1 && topk_group < n_group) {
    // group-limited routing: lane g scores group g from the selection values
    __syncwarp();
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      const int e = lane + i * 32;
      if (i < per && e < E) s_scratch[e] = sel[i];
    }
    __syncwarp();
    const int gs = E / n_group;
    float gscore = -INFINITY;
    if (lane < n_group) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = lane * gs; e < (lane + 1) * gs; ++e) {
        const float x = s_scratch[e];
        if (x > b1) { b2 = b1; b1 = x; } else if (x > b2) { b2 = x; }
      }
      gscore = group_top2 ? b1 + b2 : b1;
    }
    unsigned keep = 0;
    for (int j = 0; j < topk_group; ++j) {
      float best = gscore;
      int bi = lane < n_group ? lane : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      keep |= 1u << bi;
      if (lane == bi) gscore = -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      const int e = lane + i * 32;
      if (i < per && e < E && !((keep >> (e / gs)) & 1u)) sel[i] = -INFINITY;
    }
  }
  float wsum = 0.f;
  float my_w = 0.f;
  int my_id = 0;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      const int e = lane + i * 32;
      if (sel[i] > best) { best = sel[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    float w = 0.f;
#pragma unroll
    for (int i = 0; i < TOPK_MAX_PER_LANE; ++i) {
      if (lane + i * 32 == bi) { w = score[i]; sel[i] = -INFINITY; }
    }
    w = warp_sum(w);  // only the owner lane contributed
    wsum += w;
    if (lane == j) { my_w = w; my_id = bi; }
  }
  const float norm = (renorm && wsum > 0.f) ? 1.f / wsum : 1.f;
  const int kk = k + n_shared;
  if (lane < k) {
    ids[(long long)t * kk + lane] = my_id;
    wts[(long long)t * kk + lane] = my_w * norm * scaling;
  } else if (lane < kk) {
    ids[(long long)t * kk + lane] = E + (lane - k);
    wts[(long long)t * kk + lane] = 1.f;
  }
}

template <int VEC>
__global__ void __launch_bounds__(TOPK_THREADS)
    moe_topk_kernel(const float* __restrict__ logits, long long slab_stride, int splits,
                    const float* __restrict__ bias, int* __restrict__ ids, float* __restrict__ wts, int E, int k,
                    int n_shared, int scoring, int renorm, float scaling, int n_group, int topk_group,
                    int group_top2, const bf16* __restrict__ gx, long long ldx, const bf16* __restrict__ gw,
                    int Hd) {
  __shared__ __align__(16) float s_part[TOPK_THREADS * 4 > TOPK_MAX_E ? TOPK_THREADS * 4 : TOPK_MAX_E];
  __shared__ float s_logit[TOPK_MAX_E];
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const float* row = logits + (long long)t * E;
  const int nvec = E / VEC;
  if (gx) {
    // fused router: logits = x[t] . gate[e] (bf16 in, fp32 accumulate). The token row
    // is staged in shared memory; each warp takes two experts at a time and keeps
    // four 16-byte gate loads per expert in flight (the rows come from L2), since a
    // single dependent load chain per warp measured slower than the gate GEMM.
    bf16* s_x = reinterpret_cast<bf16*>(s_part);  // Hd <= 2 * TOPK_THREADS * 4 = 2048 elements
    const bf16* xr = gx + (long long)t * ldx;
    for (int c = tid * 8; c < Hd; c += TOPK_THREADS * 8)
      *reinterpret_cast<uint4*>(s_x + c) = *reinterpret_cast<const uint4*>(xr + c);
    __syncthreads();
    for (int e0 = (tid >> 5) * 2; e0 < E; e0 += TOPK_THREADS / 32 * 2) {
      const bf16* w0 = gw + (long long)e0 * Hd;
      const bf16* w1 = gw + (long long)min(e0 + 1, E - 1) * Hd;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c0 = lane * 8; c0 < Hd; c0 += 4 * 256) {
        uint4 p[4], q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * 256;
          if (c < Hd) {
            p[u] = __ldg(reinterpret_cast<const uint4*>(w0 + c));
            q[u] = __ldg(reinterpret_cast<const uint4*>(w1 + c));
          } else {
            p[u] = q[u] = make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * 256;
          if (c >= Hd) continue;
          float xv[8], pv[8], qv[8];
          ld_bf16x8(s_x + c, xv);
          ld_bf16x8(reinterpret_cast<const bf16*>(&p[u]), pv);
          ld_bf16x8(reinterpret_cast<const bf16*>(&q[u]), qv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc0[u] = fmaf(xv[j], pv[j], acc0[u]);
            acc1[u] = fmaf(xv[j], qv[j], acc1[u]);
          }
        }
      }
      const float l0 = warp_sum((acc0[0] + acc0[1]) + (acc0[2] + acc0[3]));
      const float l1 = warp_sum((acc1[0] + acc1[1]) + (acc1[2] + acc1[3]));
      if (lane == 0) {
        s_logit[e0] = l0;
        if (e0 + 1 < E) s_logit[e0 + 1] = l1;
      }
    }
  } else if (nvec <= TOPK_THREADS) {
    const int G = TOPK_THREADS / nvec;
    const int g = tid / nvec, v = tid - g * nvec;
    if (g < G) {
      float acc[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
#pragma unroll 4
      for (int s2 = g; s2 < splits; s2 += G) {
        const float* src = row + s2 * slab_stride + v * VEC;
        if constexpr (VEC == 4) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(src));
          acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
        } else {
          acc[0] += __ldcg(src);
        }
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) s_part[g * E + v * VEC + j] = acc[j];
    }
    __syncthreads();
    const int used = G < splits ? G : splits;
    for (int e = tid; e < E; e += TOPK_THREADS) {
      float x = 0.f;
      for (int g2 = 0; g2 < used; ++g2) x += s_part[g2 * E + e];
      s_logit[e] = x;
    }
  } else {  // more columns than threads (only E > 256 with E % 4 != 0)
    for (int e = tid; e < E; e += TOPK_THREADS) {
      float x = 0.f;
      for (int s2 = 0; s2 < splits; ++s2) x += __ldcg(row + s2 * slab_stride + e);
      s_logit[e] = x;
    }
  }
  __syncthreads();
  if (tid >= 32) return;
  route_token_warp(s_logit, s_part, t, lane, bias, ids, wts, E, k, n_shared, scoring, renorm, scaling, n_group,
                   topk_group, group_top2);
}

// Prefill-sized batches: one warp per token (8 tokens per CTA), each warp loading its
// token's logits straight into its own shared-memory row (E <= 128).
constexpr int TOPK_WARP_MAX_E = 128;
__global__ void __launch_bounds__(TOPK_THREADS)
    moe_topk_warp_kernel(const float* __restrict__ logits, long long slab_stride, int splits,
                         const float* __restrict__ bias, int* __restrict__ ids, float* __restrict__ wts, int T, int E,
                         int k, int n_shared, int scoring, int renorm, float scaling, int n_group, int topk_group,
                         int group_top2) {
  __shared__ float s_logit[TOPK_THREADS / 32][TOPK_WARP_MAX_E];
  __shared__ float s_scratch[TOPK_THREADS / 32][TOPK_WARP_MAX_E];
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (TOPK_THREADS / 32) + warp;
  if (t >= T) return;
  const float* row = logits + (long long)t * E;
  for (int e = lane; e < E; e += 32) {
    float x = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) x += __ldcg(row + s2 * slab_stride + e);
    s_logit[warp][e] = x;
  }
  __syncwarp();
  route_token_warp(s_logit[warp], s_scratch[warp], t, lane, bias, ids, wts, E, k, n_shared, scoring, renorm, scaling,
                   n_group, topk_group, group_top2);
}

void moe_topk(const float* logits, long long slab_stride, int splits, const float* bias, int* topk_ids, float* topk_w,
              int T, int E, int k, int n_shared, int scoring, int renorm, float scaling, int n_group, int topk_group,
              int group_top2, cudaStream_t s, const void* gate_x, long long ldx, const void* gate_w, int H) {
  if (T <= 0) return;
  if (E > TOPK_MAX_E) throw std::runtime_error("moe_topk: at most 512 experts");
  if (k + n_shared > 32) throw std::runtime_error("moe_topk: k + shared <= 32");
  if (n_group < 1) n_group = 1;
  if (n_group > 1) {
    if (n_group > 32 || E % n_group) throw std::runtime_error("moe_topk: n_group must divide E and be <= 32");
    if (topk_group < 1 || topk_group > n_group) throw std::runtime_error("moe_topk: 1 <= topk_group <= n_group");
    if (topk_group * (E / n_group) < k) throw std::runtime_error("moe_topk: kept groups hold fewer than k experts");
  }
  splits = splits < 1 ? 1 : splits;
  if (gate_x) {
    if (H > TOPK_THREADS * 4 * 2) throw std::runtime_error("moe_topk: fused router supports hidden <= 2048");
    if (!gate_w || H % 8 || ldx % 8 || (reinterpret_cast<uintptr_t>(gate_x) & 15) ||
        (reinterpret_cast<uintptr_t>(gate_w) & 15))
      throw std::runtime_error("moe_topk: fused router needs 16-byte aligned rows, hidden % 8 == 0");
    launch_k(moe_topk_kernel<1>, dim3(T), dim3(TOPK_THREADS), 0, s, (const float*)nullptr, 0ll, 1, bias, topk_ids,
             topk_w, E, k, n_shared, scoring, renorm, scaling, n_group, topk_group, group_top2, (const bf16*)gate_x,
             ldx, (const bf16*)gate_w, H);
    return;
  }
  if (T >= 512 && E <= TOPK_WARP_MAX_E) {  // many tokens: a warp each instead of a CTA each
    const int per_cta = TOPK_THREADS / 32;
    launch_k(moe_topk_warp_kernel, dim3((T + per_cta - 1) / per_cta), dim3(TOPK_THREADS), 0, s, logits, slab_stride,
             splits, bias, topk_ids, topk_w, T, E, k, n_shared, scoring, renorm, scaling, n_group, topk_group,
             group_top2);
    return;
  }
  const bool vec4 = E % 4 == 0 && (splits == 1 || slab_stride % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (vec4)
    launch_k(moe_topk_kernel<4>, dim3(T), dim3(TOPK_THREADS), 0, s, logits, slab_stride, splits, bias, topk_ids,
             topk_w, E, k, n_shared, scoring, renorm, scaling, n_group, topk_group, group_top2, (const bf16*)nullptr,
             0ll, (const bf16*)nullptr, 0);
  else
    launch_k(moe_topk_kernel<1>, dim3(T), dim3(TOPK_THREADS), 0, s, logits, slab_stride, splits, bias, topk_ids,
             topk_w, E, k, n_shared, scoring, renorm, scaling, n_group, topk_group, group_top2, (const bf16*)nullptr,
             0ll, (const bf16*)nullptr, 0);
}

// ---------------------------------------------------------------- align
constexpr int ALIGN_MAX_E = 1024;

// Exclusive scan of counts (and of their n-tile counts) by one warp; writes the
// row / tile prefix arrays and leaves the scatter cursors in `cursor`.
SP_DEVI void scan_counts_warp(const int* counts, int E, int bn, int* grp_rows, int* grp_tiles, int* cursor) {
  const int lane = threadIdx.x & 31;
  const int per = (E + 31) / 32;
  const int e0 = lane * per;
  int rs = 0, ts = 0;
  for (int i = 0; i < per; ++i) {
    const int e = e0 + i;
    if (e < E) { const int c = counts[e]; rs += c; ts += (c + bn - 1) / bn; }
  }
  int ri = rs, ti = ts;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, ri, o);
    const int b = __shfl_up_sync(0xffffffffu, ti, o);
    if (lane >= o) { ri += a; ti += b; }
  }
  int r = ri - rs, tt = ti - ts;
  for (int i = 0; i < per; ++i) {
    const int e = e0 + i;
    if (e < E) {
      const int c = counts[e];
      grp_rows[e] = r;
      grp_tiles[e] = tt;
      cursor[e] = r;
      r += c;
      tt += (c + bn - 1) / bn;
    }
  }
  if (lane == 31) { grp_rows[E] = ri; grp_tiles[E] = ti; }
}

__global__ void __launch_bounds__(1024) moe_align_small_kernel(const int* __restrict__ ids, int n, int k, int E,
                                                               int bn, int* __restrict__ grp_rows,
                                                               int* __restrict__ grp_tiles,
                                                               int* __restrict__ sorted_tok,
                                                               int* __restrict__ inv_pos) {
  griddep_wait();
  griddep_launch();
  __shared__ int cnt[ALIGN_MAX_E];
  __shared__ int cur[ALIGN_MAX_E];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  if (threadIdx.x < 32) scan_counts_warp(cnt, E, bn, grp_rows, grp_tiles, cur);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int pos = atomicAdd(&cur[ids[i]], 1);
    sorted_tok[pos] = i / k;
    inv_pos[i] = pos;
  }
}





// Prefill-sized layouts in three launches without contended global atomics: each CTA
// histograms its contiguous slice of the (token, slot) pairs in shared memory, one CTA
// turns the per-CTA counts into the expert offsets and each CTA's base per expert, and
// each CTA scatters its slice from those bases with shared-memory cursors. (Grid-wide
// global atomics on ~E counters measured 0.8 ms per 8,192-token chunk for count and
// scatter together.)
constexpr int ALIGN_MAX_CTAS = 128;
__global__ void __launch_bounds__(1024) moe_hist_kernel(const int* __restrict__ ids, int n, int chunk, int E,
                                                        int* __restrict__ cta_counts) {
  griddep_wait();
  griddep_launch();
  __shared__ int cnt[ALIGN_MAX_E];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int i0 = blockIdx.x * chunk, i1 = min(n, i0 + chunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cta_counts[blockIdx.x * E + e] = cnt[e];
}

__global__ void __launch_bounds__(1024) moe_bases_kernel(int* __restrict__ cta_counts, int G, int E, int bn,
                                                         int* __restrict__ grp_rows, int* __restrict__ grp_tiles) {
  griddep_wait();
  griddep_launch();
  __shared__ int tot[ALIGN_MAX_E];
  __shared__ int cur[ALIGN_MAX_E];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    for (int c = 0; c < G; ++c) t += cta_counts[c * E + e];
    tot[e] = t;
  }
  __syncthreads();
  if (threadIdx.x < 32) scan_counts_warp(tot, E, bn, grp_rows, grp_tiles, cur);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {  // counts -> each CTA's first row per expert
    int base = cur[e];
    for (int c = 0; c < G; ++c) {
      const int v = cta_counts[c * E + e];
      cta_counts[c * E + e] = base;
      base += v;
    }
  }
}

__global__ void __launch_bounds__(1024) moe_scatter_slices_kernel(const int* __restrict__ ids, int n, int chunk, int k,
                                                                  int E, const int* __restrict__ cta_bases,
                                                                  int* __restrict__ sorted_tok,
                                                                  int* __restrict__ inv_pos) {
  griddep_wait();
  griddep_launch();
  __shared__ int cur[ALIGN_MAX_E];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cur[e] = cta_bases[blockIdx.x * E + e];
  __syncthreads();
  const int i0 = blockIdx.x * chunk, i1 = min(n, i0 + chunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int pos = atomicAdd(&cur[ids[i]], 1);
    sorted_tok[pos] = i / k;
    inv_pos[i] = pos;
  }
}

int moe_align_work_ints(int E) { return (ALIGN_MAX_CTAS + 1) * E; }

int moe_align(const int* topk_ids, int T, int k, int E, int block_n, int* grp_rows, int* grp_tiles, int* sorted_tok,
              int* inv_pos, int* work, cudaStream_t s) {
  const int n = T * k;
  if (E > ALIGN_MAX_E) throw std::runtime_error("moe_align: at most 1024 experts");
  if (n <= 16384) {
    launch_k(moe_align_small_kernel, dim3(1), dim3(1024), 0, s, topk_ids, n, k, E, block_n, grp_rows, grp_tiles,
             sorted_tok, inv_pos);
    return 1;
  }
  const int G = std::min(ALIGN_MAX_CTAS, (n + 4095) / 4096);
  const int chunk = (n + G - 1) / G;
  launch_k(moe_hist_kernel, dim3(G), dim3(1024), 0, s, topk_ids, n, chunk, E, work);
  launch_k(moe_bases_kernel, dim3(1), dim3(1024), 0, s, work, G, E, block_n, grp_rows, grp_tiles);
  launch_k(moe_scatter_slices_kernel, dim3(G), dim3(1024), 0, s, topk_ids, n, chunk, k, E, (const int*)work,
           sorted_tok, inv_pos);
  return 3;
}

// ---------------------------------------------------------------- data movement
__global__ void gather_rows_kernel(const bf16* __restrict__ x, long long ldx, const int* __restrict__ idx,
                                   bf16* __restrict__ out, long long ldo, int rows, int cols) {
  griddep_wait();
  griddep_launch();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long long)idx[r] * ldx);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)r * ldo);
  for (int c = lane; c < cols / 8; c += 32) dst[c] = src[c];
}

void gather_rows(const void* x, long long ldx, const int* idx, void* out, long long ldo, int rows, int cols,
                 cudaStream_t s) {
  if (rows <= 0) return;
  if (cols % 8 || ldx % 8 || ldo % 8) throw std::runtime_error("gather_rows: 16-byte rows required");
  const int warps = 4;
  launch_k(gather_rows_kernel, dim3((rows + warps - 1) / warps), dim3(warps * 32), 0, s, (const bf16*)x, ldx, idx,
           (bf16*)out, ldo, rows, cols);
}

__global__ void silu_mul_kernel(const bf16* __restrict__ h, long long ldh, bf16* __restrict__ out, long long ldo,
                                int rows, int F) {
  griddep_wait();
  griddep_launch();
  const int per_row = F / 8;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * per_row) return;
  const int r = i / per_row, c = (i % per_row) * 8;
  float g[8], u[8];
  ld_bf16x8(h + r * ldh + c, g);
  ld_bf16x8(h + r * ldh + F + c, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) g[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
  st_bf16x8(out + r * ldo + c, g);
}

void silu_mul(const void* h, long long ldh, void* out, long long ldo, int rows, int F, cudaStream_t s) {
  if (rows <= 0) return;
  if (F % 8 || ldh % 8 || ldo % 8) throw std::runtime_error("silu_mul: 16-byte rows required");
  const long long n = (long long)rows * (F / 8);
  launch_k(silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, (const bf16*)h, ldh, (bf16*)out, ldo,
           rows, F);
}

constexpr int COMBINE_MAXK = 32;

// One thread per 8 columns of one token: blockIdx.x = token, blockIdx.y = 1024-column chunk.
__global__ void moe_combine_kernel(const bf16* __restrict__ y, long long ldy, const int* __restrict__ inv_pos,
                                   const float* __restrict__ w, const bf16* __restrict__ add, long long lda,
                                   bf16* __restrict__ out, long long ldo, int T, int k, int H) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  __shared__ int s_pos[COMBINE_MAXK];
  __shared__ float s_w[COMBINE_MAXK];
  if (threadIdx.x < k) {
    s_pos[threadIdx.x] = inv_pos[t * k + threadIdx.x];
    s_w[threadIdx.x] = w[t * k + threadIdx.x];
  }
  __syncthreads();
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= H) return;
  float acc[8];
  if (add) ld_bf16x8(add + (long long)t * lda + c, acc);
  else {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  }
  for (int j = 0; j < k; ++j) {
    float v[8];
    ld_bf16x8(y + (long long)s_pos[j] * ldy + c, v);
    const float wj = s_w[j];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += wj * v[e];
  }
  st_bf16x8(out + (long long)t * ldo + c, acc);
}

void moe_combine(const void* y, long long ldy, const int* inv_pos, const float* topk_w, const void* add,
                 long long ld_add, void* out, long long ldo, int T, int k, int H, cudaStream_t s) {
  if (T <= 0) return;
  if (k > COMBINE_MAXK) throw std::runtime_error("moe_combine: k <= 32");
  if (H % 8) throw std::runtime_error("moe_combine: hidden % 8");
  const int threads = 128;
  launch_k(moe_combine_kernel, dim3(T, (H / 8 + threads - 1) / threads), dim3(threads), 0, s, (const bf16*)y, ldy,
           inv_pos, topk_w, (const bf16*)add, ld_add, (bf16*)out, ldo, T, k, H);
}

// MoE combine fused with the next residual add + RMSNorm: one CTA per token,
//   res[t] += sum_j w[t, j] * y[inv_pos[t, j]];  out[t] = rmsnorm(res[t]) * gamma
__global__ void __launch_bounds__(256) combine_add_rmsnorm_kernel(
    const bf16* __restrict__ y, long long ldy, const int* __restrict__ inv_pos, const float* __restrict__ w,
    bf16* __restrict__ res, const bf16* __restrict__ gamma, bf16* __restrict__ out, long long ldo, int k, int H,
    float eps, const bf16* __restrict__ sh, long long ldsh, int n_sh, int T) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  __shared__ int s_pos[COMBINE_MAXK];
  __shared__ float s_w[COMBINE_MAXK];
  __shared__ float part[8];
  if (threadIdx.x < k) {
    s_pos[threadIdx.x] = inv_pos[t * k + threadIdx.x];
    s_w[threadIdx.x] = w[t * k + threadIdx.x];
  }
  __syncthreads();
  bf16* rr = res + (long long)t * H;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // four rows' loads in flight before their sums (the rows are scattered in y);
      // the sum keeps the j order, so results do not change with the grouping
      int j = 0;
      for (; j + 4 <= k; j += 4) {
        float yv[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) ld_bf16x8(y + (long long)s_pos[j + u] * ldy + c, yv[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += s_w[j + u] * yv[u][e];
      }
      for (; j < k; ++j) {
        float yv[8];
        ld_bf16x8(y + (long long)s_pos[j] * ldy + c, yv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += s_w[j] * yv[e];
      }
      // shared experts computed apart (rows s * T + t of sh, weight 1), after the routed ones
      for (int q = 0; q < n_sh; ++q) {
        float yv[8];
        ld_bf16x8(sh + ((long long)q * T + t) * ldsh + c, yv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += yv[e];
      }
      float r[8];
      ld_bf16x8(rr + c, r);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[i][e] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(acc[e])) + r[e]));
      st_bf16x8(rr + c, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float inv = rsqrtf(tot / H + eps);
  bf16* orow = out + (long long)t * ldo;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float g[8];
      ld_bf16x8(gamma + c, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] * inv * g[e];
      st_bf16x8(orow + c, v[i]);
    }
  }
}

void combine_add_rmsnorm(const void* y, long long ldy, const int* inv_pos, const float* topk_w, void* residual,
                         const void* gamma, void* out, long long ldo, int T, int k, int H, float eps, cudaStream_t s,
                         const void* shared, long long ld_shared, int n_shared) {
  if (T <= 0) return;
  if (k > COMBINE_MAXK) throw std::runtime_error("combine_add_rmsnorm: k <= 32");
  if (H % 8 || H > 8192) throw std::runtime_error("combine_add_rmsnorm: hidden % 8, <= 8192");
  launch_k(combine_add_rmsnorm_kernel, dim3(T), dim3(256), 0, s, (const bf16*)y, ldy, inv_pos, topk_w,
           (bf16*)residual, (const bf16*)gamma, (bf16*)out, ldo, k, H, eps, (const bf16*)shared, ld_shared,
           shared ? n_shared : 0, T);
}

void kernel_attrs_moe(std::vector<KernelAttr>& out) {
  push_kernel_attr(out, "moe_topk_kernel<4>", moe_topk_kernel<4>);
  push_kernel_attr(out, "moe_topk_kernel<1>", moe_topk_kernel<1>);
  push_kernel_attr(out, "moe_align_small_kernel", moe_align_small_kernel);
}

}  // namespace sp
