// DeepSeek sparse attention (DSA) token selection for decode, sm_100a.
//
// For a sequence b with index query heads q[b, h, :] (Hi heads x 128), head
// weights w[b, h] and one 128-wide index key k[s, :] per cached token s, the
// index score is
//
//   score[b, s] = sum_h w[b, h] * relu(q[b, h, :] . k[s, :])
//
// and attention reads only the `topk` highest-scoring tokens. The raw products
// q . k for all heads and tokens form a GEMM and run on the tcgen05 GEMM (keys
// gathered from the paged index-key cache into a dense block first); this file
// holds the rest:
//
//   paged_slots        cache slot of each (sequence, position) through the block
//                      table (contiguous positions, or a list of positions)
//   dsa_topk           per sequence: the weighted relu head reduce into scores,
//                      then an exact radix select of the topk largest (four 8-bit
//                      digit passes over order-preserving keys; ties at the
//                      threshold filled in index order of discovery), then the
//                      selected positions sorted ascending (bitonic sort in
//                      shared memory) so the KV gather reads in order
//
// Reference: PHASE_DSA_SELECTION, DSA_SCORE_TILE_ROWS and the selected-token
// fields of crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h
// (:74, :445-478); the kernels are this framework's own.
#include <cuda_runtime.h>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

__global__ void paged_slots_kernel(const int* __restrict__ block_table, int max_blocks, const int* __restrict__ lens,
                                   const int* __restrict__ positions, int rows, int block_size,
                                   int* __restrict__ slots) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const int n = lens[b];
  int slot = 0;  // rows past the length read slot 0 (masked by the consumer)
  if (i < n) {
    const int pos = positions ? positions[(long long)b * rows + i] : i;
    const int blk = pos / block_size;
    if (pos >= 0 && blk < max_blocks)
      slot = block_table[(long long)b * max_blocks + blk] * block_size + pos % block_size;
  }
  slots[(long long)b * rows + i] = slot;
}

void paged_slots(const int* block_table, int max_blocks, const int* lens, const int* positions, int B, int rows,
                 int block_size, int* slots, cudaStream_t s) {
  if (B <= 0 || rows <= 0) return;
  launch_k(paged_slots_kernel, dim3((rows + 255) / 256, B), dim3(256), 0, s, block_table, max_blocks, lens,
           positions, rows, block_size, slots);
}

namespace {
constexpr int TOPK_THREADS = 1024;
constexpr int MAX_TOPK = 2048;

SP_DEVI uint32_t order_key(float x) {  // larger float -> larger key
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
}  // namespace

// One CTA per sequence. raw: [B, Hi, rows] q.k products; scores: [B, rows] scratch.
__global__ void __launch_bounds__(TOPK_THREADS) dsa_topk_kernel(const float* __restrict__ raw,
                                                                const float* __restrict__ w, int Hi, int rows,
                                                                const int* __restrict__ lens, int topk,
                                                                float* __restrict__ scores, int* __restrict__ out,
                                                                int* __restrict__ counts) {
  griddep_wait();
  griddep_launch();
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_need, s_above, s_eq;
  __shared__ int sel[MAX_TOPK];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int n = min(lens[b], rows);
  const float* rb = raw + (long long)b * Hi * rows;
  float* sc = scores + (long long)b * rows;
  // ---- weighted relu head reduce
  for (int s = tid; s < n; s += TOPK_THREADS) {
    float acc = 0.f;
    for (int h = 0; h < Hi; ++h) acc += w[(long long)b * Hi + h] * fmaxf(rb[(long long)h * rows + s], 0.f);
    sc[s] = acc;
  }
  __syncthreads();
  const int k = min(topk, n);
  if (tid == 0) counts[b] = k;
  int* ob = out + (long long)b * topk;
  if (k == n) {  // everything is selected: positions in order
    for (int i = tid; i < topk; i += TOPK_THREADS) ob[i] = i < n ? i : -1;
    return;
  }
  // ---- radix select of the k-th largest order key, 8 bits at a time from the top
  if (tid == 0) {
    s_prefix = 0;
    s_need = (uint32_t)k;
  }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += TOPK_THREADS) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    const uint32_t mask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int s = tid; s < n; s += TOPK_THREADS) {
      const uint32_t key = order_key(sc[s]);
      if ((key & mask) == (prefix & mask)) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = s_need, acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= need) break;
        acc += hist[d];
      }
      s_prefix = prefix | (uint32_t(d) << shift);
      s_need = need - acc;  // how many with exactly this digit prefix are still needed
    }
    __syncthreads();
  }
  // ---- collect: every key above the threshold, then `need` keys equal to it
  const uint32_t thr = s_prefix;
  const uint32_t need_eq = s_need;
  if (tid == 0) {
    s_above = 0;
    s_eq = 0;
  }
  __syncthreads();
  const uint32_t n_above = (uint32_t)k - need_eq;
  for (int s = tid; s < n; s += TOPK_THREADS) {
    const uint32_t key = order_key(sc[s]);
    if (key > thr) {
      const uint32_t j = atomicAdd(&s_above, 1u);
      if (j < n_above) sel[j] = s;
    } else if (key == thr) {
      const uint32_t j = atomicAdd(&s_eq, 1u);
      if (j < need_eq) sel[n_above + j] = s;
    }
  }
  __syncthreads();
  // ---- bitonic sort of the k positions ascending (padded to a power of two)
  int P = 1;
  while (P < k) P <<= 1;
  for (int i = k + tid; i < P; i += TOPK_THREADS) sel[i] = 0x7fffffff;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += TOPK_THREADS) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const int a = sel[i], c = sel[j];
          if ((a > c) == up) {
            sel[i] = c;
            sel[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < topk; i += TOPK_THREADS) ob[i] = i < k ? sel[i] : -1;
}

void dsa_topk(const float* raw, const float* w, int B, int Hi, int rows, const int* lens, int topk, float* scores,
              int* out, int* counts, cudaStream_t s) {
  if (B <= 0) return;
  if (topk <= 0 || topk > MAX_TOPK) throw std::runtime_error("dsa_topk: topk must be 1..2048");
  launch_k(dsa_topk_kernel, dim3(B), dim3(TOPK_THREADS), 0, s, raw, w, Hi, rows, lens, topk, scores, out, counts);
}

}  // namespace sp
