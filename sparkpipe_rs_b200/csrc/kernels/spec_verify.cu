// Speculative-decode verify kernels of the serving engine, sm_100a.
//
// Row arrays of a verify round are row-major by draft depth / tree row: row
// j * B + b belongs to batch lane b (B = padded lanes). `tok` holds each row's
// input token, `tgt` the verifier's greedy token after it.
//
//  * spec_chain_commit — chain of drafts: lane b accepts the longest prefix of
//                        its drafts t_1..t_d (d = its draft budget) that the
//                        verifier agrees with, or for benchmarks a seeded
//                        Bernoulli(p) chain keyed by (seed, lane key, position,
//                        depth); commits the accepted drafts and the verifier's
//                        token after them.
//  * mtp_tree_commit   — the fixed MTP draft tree (5 candidates, 6 rows: row r
//                        holds candidate r - 1; rows 3 and 5 are the alternate
//                        leaves of depth 2 and 3): walks from the input row to
//                        the child whose candidate equals the verifier's token,
//                        commits the path's candidates and the verifier's token
//                        at its end, and, when the path ends on an alternate
//                        leaf, moves that leaf's KV from its shadow slot to the
//                        primary position's slot in every layer of the cache.
//  * top2_rows         — the two largest logits of each row (ties to the lower
//                        id), written to two separate id arrays: the tree
//                        drafter's primary and alternate candidates.
//
// Reference: the MTP tree and its resolution (crates/spark-sched/src/work_control.rs:
// 107-253, crates/spark-serve/src/request_api/speculation.rs:211-254, 807-882).
#include <cuda_runtime.h>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {
SP_DEVI uint64_t mix(uint64_t z) {  // SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014)
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
SP_DEVI float unit(uint64_t seed, uint64_t key, uint64_t pos, uint64_t depth) {
  const uint64_t h = mix(seed ^ mix(key ^ mix(pos ^ mix(depth))));
  return ((h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}

// tree rows: parent row, depth, first child row, child count (row r's token is candidate r - 1)
__constant__ int8_t kTreeParent[6] = {0, 0, 1, 1, 2, 2};
__constant__ int8_t kTreeDepth[6] = {0, 1, 2, 2, 3, 3};
__constant__ int8_t kTreeChild0[6] = {1, 2, 4, 0, 0, 0};
__constant__ int8_t kTreeChildren[6] = {1, 2, 2, 0, 0, 0};
constexpr int kTreeRows = 6;
}  // namespace

__global__ void spec_chain_commit_kernel(const int* __restrict__ tok, const int* __restrict__ tgt,
                                         const int* __restrict__ ctx, const int* __restrict__ pos,
                                         const int* __restrict__ budget, const unsigned long long* __restrict__ keys,
                                         int B, int L, float p_accept, uint64_t seed, int* __restrict__ committed,
                                         int* __restrict__ counts) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int* out = committed + (long long)b * (L + 1);
  if (ctx[b] == 0) {  // idle lane
    counts[b] = 0;
    for (int i = 0; i <= L; ++i) out[i] = -1;
    return;
  }
  const int d = min(max(budget[b], 0), L);
  int a = 0;
  for (; a < d; ++a) {
    bool ok;
    if (p_accept > 0.f) ok = unit(seed, keys[b], (uint64_t)pos[b], (uint64_t)a) < p_accept;
    else ok = tok[(a + 1) * B + b] == tgt[a * B + b];
    if (!ok) break;
  }
  for (int i = 0; i <= L; ++i) out[i] = i < a ? tok[(i + 1) * B + b] : (i == a ? tgt[a * B + b] : -1);
  counts[b] = a + 1;
}

void spec_chain_commit(const int* tok, const int* tgt, const int* ctx, const int* pos, const int* budget,
                       const unsigned long long* keys, int B, int L, float p_accept, unsigned long long seed,
                       int* committed, int* counts, cudaStream_t s) {
  if (B <= 0) return;
  launch_k(spec_chain_commit_kernel, dim3((B + 127) / 128), dim3(128), 0, s, tok, tgt, ctx, pos, budget, keys, B, L,
           p_accept, (uint64_t)seed, committed, counts);
}

// One CTA per lane: thread 0 resolves the path, then the CTA moves the accepted
// alternate leaf's KV row (row_elems bf16, 16-byte chunks) in every layer.
__global__ void __launch_bounds__(128) mtp_tree_commit_kernel(const int* __restrict__ tok, const int* __restrict__ tgt,
                                                              const int* __restrict__ ctx,
                                                              const int* __restrict__ slots, int B,
                                                              bf16* __restrict__ cache, long long layer_stride,
                                                              int layers, int row_elems, int* __restrict__ committed,
                                                              int* __restrict__ counts, int* __restrict__ paths,
                                                              float* __restrict__ aux, long long aux_layer_stride,
                                                              int aux_row) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x;
  __shared__ int s_path;
  if (threadIdx.x == 0) {
    int* out = committed + (long long)b * kTreeRows;
    if (ctx[b] == 0) {  // idle lane
      counts[b] = 0;
      paths[b] = 0;
      for (int i = 0; i < kTreeRows; ++i) out[i] = -1;
      s_path = 0;
    } else {
      int row = 0;
      for (bool moved = true; moved;) {
        moved = false;
        const int want = tgt[row * B + b];
        for (int c = 0; c < kTreeChildren[row]; ++c) {
          const int child = kTreeChild0[row] + c;
          if (tok[child * B + b] == want) {
            row = child;
            moved = true;
            break;
          }
        }
      }
      const int depth = kTreeDepth[row];
      // the path's candidates from depth 1 down to the end row, then the verifier's token there
      int r = row;
      for (int k = depth - 1; k >= 0; --k) {
        out[k] = tok[r * B + b];
        r = kTreeParent[r];
      }
      out[depth] = tgt[row * B + b];
      for (int i = depth + 1; i < kTreeRows; ++i) out[i] = -1;
      counts[b] = depth + 1;
      paths[b] = row;
      s_path = row;
    }
  }
  __syncthreads();
  const int path = s_path;
  if (path != 3 && path != 5) return;
  // alternate leaf accepted: its shadow row becomes the primary row of its depth
  const int src = slots[path * B + b], dst = slots[(path == 3 ? 2 : 4) * B + b];
  if (src < 0 || dst < 0) return;
  const int chunks = row_elems / 8;
  for (int i = threadIdx.x; i < layers * chunks; i += blockDim.x) {
    const int l = i / chunks, c = i - l * chunks;
    const uint4* s4 = reinterpret_cast<const uint4*>(cache + l * layer_stride + (long long)src * row_elems) + c;
    uint4* d4 = reinterpret_cast<uint4*>(cache + l * layer_stride + (long long)dst * row_elems) + c;
    *d4 = *s4;
  }
  // the row's side array (the fp8 cache's block scales), word by word
  for (int i = threadIdx.x; aux && i < layers * aux_row; i += blockDim.x) {
    const int l = i / aux_row, c = i - l * aux_row;
    aux[l * aux_layer_stride + (long long)dst * aux_row + c] = aux[l * aux_layer_stride + (long long)src * aux_row + c];
  }
}

void mtp_tree_commit(const int* tok, const int* tgt, const int* ctx, const int* slots, int B, void* cache,
                     long long layer_stride, int layers, int row_elems, int* committed, int* counts, int* paths,
                     cudaStream_t s, float* aux, long long aux_layer_stride, int aux_row) {
  if (B <= 0) return;
  if (row_elems % 8 || layer_stride % 8) throw std::runtime_error("mtp_tree_commit: 16-byte KV rows required");
  launch_k(mtp_tree_commit_kernel, dim3(B), dim3(128), 0, s, tok, tgt, ctx, slots, B, static_cast<bf16*>(cache),
           layer_stride, layers, row_elems, committed, counts, paths, aux, aux_layer_stride, aux_row);
}

namespace {
// (va, ia) ranks before (vb, ib): larger logit, then lower id
SP_DEVI bool before(float va, int ia, float vb, int ib) { return va > vb || (va == vb && ia < ib); }
SP_DEVI void insert2(float v, int i, float& v0, int& i0, float& v1, int& i1) {
  if (before(v, i, v0, i0)) {
    v1 = v0; i1 = i0; v0 = v; i0 = i;
  } else if (before(v, i, v1, i1)) {
    v1 = v; i1 = i;
  }
}
}  // namespace

__global__ void __launch_bounds__(1024) top2_rows_kernel(const bf16* __restrict__ logits, long long ldl, int V,
                                                          int* __restrict__ out0, int* __restrict__ out1) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const bf16* lr = logits + (long long)row * ldl;
  float v0 = -INFINITY, v1 = -INFINITY;
  int i0 = 0x7fffffff, i1 = 0x7fffffff;
  if ((V % 8 == 0) && (ldl % 8 == 0)) {
    for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
      float v[8];
      ld_bf16x8(lr + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) insert2(v[e], c + e, v0, i0, v1, i1);
    }
  } else {
    for (int c = threadIdx.x; c < V; c += blockDim.x) insert2(__bfloat162float(lr[c]), c, v0, i0, v1, i1);
  }
  // butterfly: each step merges the pairs of two disjoint id subsets
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a0 = __shfl_xor_sync(0xffffffffu, v0, o), a1 = __shfl_xor_sync(0xffffffffu, v1, o);
    const int b0 = __shfl_xor_sync(0xffffffffu, i0, o), b1 = __shfl_xor_sync(0xffffffffu, i1, o);
    insert2(a0, b0, v0, i0, v1, i1);
    insert2(a1, b1, v0, i0, v1, i1);
  }
  __shared__ float sv[2][32];
  __shared__ int si[2][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[0][w] = v0; si[0][w] = i0; sv[1][w] = v1; si[1][w] = i1;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    v0 = lane < nw ? sv[0][lane] : -INFINITY;
    i0 = lane < nw ? si[0][lane] : 0x7fffffff;
    v1 = lane < nw ? sv[1][lane] : -INFINITY;
    i1 = lane < nw ? si[1][lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float a0 = __shfl_xor_sync(0xffffffffu, v0, o), a1 = __shfl_xor_sync(0xffffffffu, v1, o);
      const int b0 = __shfl_xor_sync(0xffffffffu, i0, o), b1 = __shfl_xor_sync(0xffffffffu, i1, o);
      insert2(a0, b0, v0, i0, v1, i1);
      insert2(a1, b1, v0, i0, v1, i1);
    }
    if (lane == 0) {
      out0[row] = i0;
      out1[row] = i1;
    }
  }
}

void top2_rows(const void* logits, long long ldl, int T, int V, int* out0, int* out1, cudaStream_t s) {
  if (T <= 0) return;
  if (V < 2) throw std::runtime_error("top2_rows: needs two columns");
  launch_k(top2_rows_kernel, dim3(T), dim3(1024), 0, s, (const bf16*)logits, ldl, V, out0, out1);
}

}  // namespace sp
