// Token sampling, embedding gather and speculative-decode verification, sm_100a.
//
//  * sample_tokens — greedy argmax (temperature <= 0) or Gumbel-max sampling
//                    (argmax of logits / T + Gumbel noise). Noise comes from a
//                    SplitMix64 hash (Steele, Lea & Flood, OOPSLA 2014) of
//                    (seed, offset, row, column), so a replay with the same seed
//                    reproduces the same tokens.
//  * embedding     — token id -> bf16 row.
//  * spec_verify   — accept the longest draft prefix that matches the
//                    verifier's tokens (or, for benchmarking, a seeded
//                    Bernoulli(p) chain), emit the committed tokens (accepted
//                    drafts + one verifier token).
//
// Reference: RESTRICTED_LOGITS / FUSED_FINAL_TOKEN_TAIL and MTP_VERIFY phases
// of crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:445-460, 645-671,
// and the accept/commit rule of crates/spark-serve/src/request_api/speculation.rs:211-254.
#include <cuda_runtime.h>

#include <algorithm>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

SP_DEVI uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
SP_DEVI float uniform01(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  const uint64_t h = splitmix64(seed ^ splitmix64(a ^ splitmix64(b ^ splitmix64(c))));
  return ((h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}

// With per-row parameters (row_temp != nullptr) each row has its own temperature
// and noise key, and the noise does not depend on the row's place in the batch:
// the same request draws the same tokens however it is batched.
__global__ void sample_kernel(const bf16* __restrict__ logits, long long ldl, int V, float temp, uint64_t seed,
                              uint64_t offset, int* __restrict__ out_ids, float* __restrict__ out_logit,
                              const float* __restrict__ row_temp, const unsigned long long* __restrict__ row_key) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  uint64_t hrow = row;
  if (row_temp) {
    temp = row_temp[row];
    seed = row_key[row];
    offset = 0;
    hrow = 0;
  }
  const bf16* lr = logits + (long long)row * ldl;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const float inv_t = temp > 0.f ? 1.f / temp : 0.f;
  const bool vec = (V % 8 == 0) && (ldl % 8 == 0);
  if (vec) {
    for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
      float v[8];
      ld_bf16x8(lr + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float s = v[e];
        if (temp > 0.f) s = s * inv_t - __logf(-__logf(uniform01(seed, offset, hrow, c + e)));
        if (s > best) { best = s; bi = c + e; }
      }
    }
  } else {
    for (int c = threadIdx.x; c < V; c += blockDim.x) {
      float s = __bfloat162float(lr[c]);
      if (temp > 0.f) s = s * inv_t - __logf(-__logf(uniform01(seed, offset, hrow, c)));
      if (s > best) { best = s; bi = c; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) {
      out_ids[row] = bi;
      if (out_logit) out_logit[row] = __bfloat162float(lr[bi]);
    }
  }
}

void sample_tokens(const void* logits, long long ldl, int T, int V, float temperature, unsigned long long seed,
                   unsigned long long offset, int* out_ids, float* out_logit, const float* row_temp,
                   const unsigned long long* row_key, cudaStream_t s) {
  if (T <= 0) return;
  launch_k(sample_kernel, dim3(T), dim3(1024), 0, s, (const bf16*)logits, ldl, V, temperature, (uint64_t)seed,
           (uint64_t)offset, out_ids, out_logit, row_temp, row_key);
}

// Fills the first n rows of a decode step's token ids from the previous step's
// sampled tokens: on entry ids[i] holds the previous step's row index.
__global__ void gather_prev_tokens_kernel(int* __restrict__ ids, const int* __restrict__ prev, int n, int prev_rows) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = ids[i];
  ids[i] = (r >= 0 && r < prev_rows) ? prev[r] : 0;
}

void gather_prev_tokens(int* ids, const int* prev, int n, int prev_rows, cudaStream_t s) {
  if (n <= 0) return;
  launch_k(gather_prev_tokens_kernel, dim3((n + 127) / 128), dim3(128), 0, s, ids, prev, n, prev_rows);
}

__global__ void embedding_kernel(const bf16* __restrict__ table, long long ld, const int* __restrict__ ids,
                                 bf16* __restrict__ out, long long ldo, int T, int H) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const uint4* src = reinterpret_cast<const uint4*>(table + (long long)ids[t] * ld);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * ldo);
  for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

void embedding(const void* table, long long ld, const int* ids, void* out, long long ldo, int T, int H,
               cudaStream_t s) {
  if (T <= 0) return;
  if (H % 8 || ld % 8 || ldo % 8) throw std::runtime_error("embedding: 16-byte rows required");
  const int warps = 8;
  launch_k(embedding_kernel, dim3((T + warps - 1) / warps), dim3(warps * 32), 0, s, (const bf16*)table, ld, ids,
           (bf16*)out, ldo, T, H);
}

__global__ void spec_verify_kernel(const int* __restrict__ draft, const int* __restrict__ target, int B, int L,
                                   float p_accept, uint64_t seed, uint64_t offset, int* __restrict__ accepted,
                                   int* __restrict__ committed) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int a = 0;
  for (; a < L; ++a) {
    bool ok;
    if (p_accept > 0.f) ok = uniform01(seed, offset, b, a) < p_accept;
    else ok = draft[b * L + a] == target[b * (L + 1) + a];
    if (!ok) break;
  }
  accepted[b] = a;
  // committed = accepted drafts followed by the verifier's token at the first
  // rejected position (or the bonus token after a fully accepted chain)
  for (int i = 0; i <= L; ++i) {
    int tok = -1;
    if (i < a) tok = draft[b * L + i];
    else if (i == a) tok = target[b * (L + 1) + a];
    committed[b * (L + 1) + i] = tok;
  }
}

void spec_verify(const int* draft, const int* target, int B, int L, float forced_accept_p, unsigned long long seed,
                 unsigned long long offset, int* accepted, int* committed, cudaStream_t s) {
  if (B <= 0) return;
  launch_k(spec_verify_kernel, dim3((B + 127) / 128), dim3(128), 0, s, draft, target, B, L, forced_accept_p,
           (uint64_t)seed, (uint64_t)offset, accepted, committed);
}

// End of one speculative round, one thread per sequence b. Row arrays are
// j-major (row j*B + b, j = 0..L): tok_rows holds the round's inputs (t_0 = the
// last committed token, t_j = draft token j), tgt_rows the verifier's greedy
// token after each input. Acceptance is the longest draft prefix the verifier
// agrees with, or (p_accept > 0, benchmarking) a seeded Bernoulli(p) chain keyed
// by (seed, position of t_0, b, j). Writes the committed tokens (accepted drafts,
// then the verifier's token at the first rejection), and advances the row arrays
// in place for the next round: t_0 <- that verifier token, positions / context
// lengths / cache slots of rows j = new position + j. Context lengths are clamped
// to the block table, so a sequence that ran out of blocks never reads past it.
__global__ void spec_finish_kernel(int* __restrict__ tok_rows, const int* __restrict__ tgt_rows, int B, int L,
                                   float p_accept, uint64_t seed, int* __restrict__ pos_rows,
                                   int* __restrict__ ctx_rows, int* __restrict__ slot_rows,
                                   const int* __restrict__ block_table, int max_blocks, int block_size,
                                   int* __restrict__ accepted, int* __restrict__ committed,
                                   unsigned long long* __restrict__ total_committed) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int p0 = pos_rows[b];
  if (p0 < 0) return;  // idle row
  int a = 0;
  for (; a < L; ++a) {
    bool ok;
    if (p_accept > 0.f) ok = uniform01(seed, (uint64_t)p0, b, a) < p_accept;
    else ok = tok_rows[(a + 1) * B + b] == tgt_rows[a * B + b];
    if (!ok) break;
  }
  for (int i = 0; i <= L; ++i) {
    int t = -1;
    if (i < a) t = tok_rows[(i + 1) * B + b];
    else if (i == a) t = tgt_rows[a * B + b];
    committed[b * (L + 1) + i] = t;
  }
  accepted[b] = a;
  if (total_committed) atomicAdd(total_committed, (unsigned long long)(a + 1));
  tok_rows[b] = tgt_rows[a * B + b];
  const int np = p0 + a + 1;
  const int cap = max_blocks * block_size;
  for (int j = 0; j <= L; ++j) {
    const int p = np + j;
    const int blk = p / block_size;
    pos_rows[j * B + b] = p;
    ctx_rows[j * B + b] = min(p + 1, cap);
    slot_rows[j * B + b] = blk < max_blocks ? block_table[(long long)b * max_blocks + blk] * block_size + p % block_size
                                            : -1;
  }
}

void spec_finish(int* tok_rows, const int* tgt_rows, int B, int L, float p_accept, unsigned long long seed,
                 int* pos_rows, int* ctx_rows, int* slot_rows, const int* block_table, int max_blocks,
                 int block_size, int* accepted, int* committed, unsigned long long* total_committed, cudaStream_t s) {
  if (B <= 0) return;
  launch_k(spec_finish_kernel, dim3((B + 127) / 128), dim3(128), 0, s, tok_rows, tgt_rows, B, L, p_accept,
           (uint64_t)seed, pos_rows, ctx_rows, slot_rows, block_table, max_blocks, block_size, accepted, committed,
           total_committed);
}

// Paged KV blocks <-> a contiguous staging buffer, for moving blocks between the
// device cache [layers][slots][row] and a host tier. One CTA per (block, layer)
// copies block_size rows of `row` bf16 with 16-byte accesses; the staging layout is
// [n][layers][block_size][row], so a batch of blocks moves to or from pinned host
// memory in one copy.
__global__ void __launch_bounds__(256) kv_blocks_copy_kernel(bf16* __restrict__ cache, long long layer_stride,
                                                              const int* __restrict__ blocks, bf16* __restrict__ staging,
                                                              int layers, int block_size, int row, int to_staging) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x / layers, l = blockIdx.x - (blockIdx.x / layers) * layers;
  const long long n8 = (long long)block_size * row / 8;
  uint4* c = reinterpret_cast<uint4*>(cache + l * layer_stride + (long long)blocks[i] * block_size * row);
  uint4* st = reinterpret_cast<uint4*>(staging + ((long long)i * layers + l) * block_size * row);
  for (long long k = threadIdx.x; k < n8; k += blockDim.x) {
    if (to_staging) st[k] = c[k];
    else c[k] = st[k];
  }
}

void kv_blocks_copy(void* cache, long long layer_stride, const int* blocks, int n, void* staging, int layers,
                    int block_size, int row, int to_staging, cudaStream_t s) {
  if (n <= 0) return;
  if ((long long)block_size * row % 8 || layer_stride % 8) throw std::runtime_error("kv_blocks_copy: 16-byte rows");
  launch_k(kv_blocks_copy_kernel, dim3((unsigned)(n * layers)), dim3(256), 0, s, static_cast<bf16*>(cache),
           layer_stride, blocks, static_cast<bf16*>(staging), layers, block_size, row, to_staging);
}

// Phase clock: one thread stamps the device's global timer (ns) into slot `slot`
// of a step's clock array and adds the time since slot `prev`'s stamp to the
// phase's running total. Stream-ordered with the kernels around it (it waits for
// its predecessor before reading the timer, and with programmatic launch every
// predecessor has waited for its own), so the totals are the device time of the
// phases between marks, accumulated over layers and steps.
__global__ void phase_mark_kernel(unsigned long long* stamps, unsigned long long* totals, int slot, int prev) {
  griddep_wait();
  griddep_launch();
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (totals && prev >= 0) totals[slot] += t - stamps[prev];
  stamps[slot] = t;
}

void phase_mark(unsigned long long* stamps, unsigned long long* totals, int slot, int prev, cudaStream_t s) {
  launch_k(phase_mark_kernel, dim3(1), dim3(1), 0, s, stamps, totals, slot, prev);
}

// Feeds a decode step's sampled tokens back as the next step's inputs: token id,
// position + 1, context length + 1 and the cache slot of the new position
// (from the block table; -1 once the table is exhausted). Rows with a zero
// context length are idle and left untouched.
__global__ void decode_advance_kernel(const int* __restrict__ out_ids, int* __restrict__ ids, int* __restrict__ pos,
                                      int* __restrict__ ctx, int* __restrict__ slots,
                                      const int* __restrict__ block_table, int max_blocks, int B, int block_size) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || ctx[b] == 0) return;
  ids[b] = out_ids[b];
  const int p = pos[b] + 1;
  pos[b] = p;
  ctx[b] = p + 1;
  const int blk = p / block_size;
  slots[b] = blk < max_blocks ? block_table[(long long)b * max_blocks + blk] * block_size + p % block_size : -1;
}

void decode_advance(const int* out_ids, int* ids, int* pos, int* ctx, int* slots, const int* block_table,
                    int max_blocks, int B, int block_size, cudaStream_t s) {
  if (B <= 0) return;
  launch_k(decode_advance_kernel, dim3((B + 127) / 128), dim3(128), 0, s, out_ids, ids, pos, ctx, slots, block_table,
           max_blocks, B, block_size);
}

}  // namespace sp
