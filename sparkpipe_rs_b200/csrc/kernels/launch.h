// Host-side launch interfaces of the sm_100a kernels. Plain C++ (no torch
// headers) so the .cu translation units compile quickly; ops.cpp binds these
// to torch tensors.
#pragma once
#include <string>
#include <vector>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sp {

// D[m, n] = sum_k A[m, k] * B[n, k]; see gemm_tcgen05.cu for the modes.
// Tensor-parallel operands of a GEMM over peer memory (gemm_tcgen05.cu): a
// reduce-scatter epilogue into the owner ranks' slots and/or an all-gathered B
// operand read from this rank's tagged-word region.
struct TpGemm {
  unsigned long long base[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // rank buffer bases (peer pointers)
  long long rs_off = 0;          // reduce-scatter region: [2][world * splits][rows][M] words
  int rs = 0, rank = 0, world = 1, rows = 0;
  const void* ag_flags = nullptr;  // all-gather row flags of this rank: [2][world * rows] tags (B = the region)
  const int64_t* epoch = nullptr;
  int layer = 0, layers_per_step = 2;
  long long budget = 4000000000ll;
  int max_splits = 4;
};

// Expert-parallel combine fused into a grouped GEMM's epilogue: output row p goes to
// rank comb_dst[p] >> 20, combine slot comb_dst[p] & 0xFFFFF, as tagged bf16 pairs
// (the layout ep.cu's combine reads; see parallel/expert_parallel.py for the regions).
struct EpComb {
  unsigned long long base[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  long long comb_off = 0;
  int cap = 0, kk = 0, H = 0, layers_per_step = 2;
  const int* comb_dst = nullptr;
  const int64_t* epoch = nullptr;
  int layer = 0;
};

struct GemmLaunch {
  const void* A = nullptr;
  long long a_rows = 0, a_cols = 0, lda = 0;  // 2-D view of A as stored (elements)
  const void* B = nullptr;
  long long b_rows = 0, b_cols = 0, ldb = 0;
  void* D = nullptr;
  long long ldd = 0, d_batch_stride = 0;
  int M = 0, N = 0, K = 0, batch = 1;
  int a_row0 = 0, a_batch_rows = 0, a_k0 = 0, a_batch_k = 0;
  int b_row0 = 0, b_batch_rows = 0, b_k0 = 0, b_batch_k = 0;
  int trans_out = 0;  // 1: write D^T, i.e. element (m, n) to D[n * ldd + m]
  int out_f32 = 0;
  int splits = 0;     // split-K cluster size; 0 = automatic, 1 = off
  int block_n = 0;    // 0 = automatic
  int grouped = 0;
  const int* grp_rows = nullptr;   // [num_groups + 1] B-row prefix offsets
  const int* grp_tiles = nullptr;  // [num_groups + 1] n-tile prefix counts (for block_n)
  int num_groups = 0;
  int a_evict_first = 0;
  // grouped (weight-major) only: grp_rows / grp_tiles were written at least two launches
  // back, so the producer may read the tile schedule and stream the first weight tiles
  // before the PDL wait (the launch right before it has itself waited for their writer)
  int sched_early = 0;
  int swiglu = 0;  // grouped only: fused silu(gate) * up epilogue, output [rows, M / 2]
  float* ws = nullptr;        // split-K partial workspace (fp32 slabs)
  long long ws_floats = 0;
  int slab_out = 0;           // split-K: leave the partial slabs (dense [rows][cols] fp32) for the consumer
  int* err = nullptr;
  int num_sms = 148;
  cudaStream_t stream = 0;
  const TpGemm* tp = nullptr;
  const EpComb* ep = nullptr;  // grouped only: send the output rows to their source ranks
};
// Returns the number of kernels launched, or -splits when the result was left as
// `splits` fp32 slabs in g.ws (slab_out requested and K was split).
int gemm_bf16(const GemmLaunch& g);
void make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, long long rows,
                  long long cols, long long ld, int box_rows, int box_cols);
void make_tmap_2d_swizzle(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, long long rows,
                          long long cols, long long ld, int box_rows, int box_cols, CUtensorMapSwizzle swizzle);
// out[r, c] = sum_s ws[s][r][c] for `splits` dense fp32 slabs [rows, cols] `stride` apart (cols % 4 == 0).
void split_reduce(const float* ws, long long stride, int splits, int rows, int cols, void* out, long long ldo,
                  int out_f32, cudaStream_t s);

// ---- tensor parallelism over peer memory (tp.cu)
struct TpArgs {
  unsigned long long base[8];  // rank buffer bases (peer pointers)
  long long rs_off;            // RS region: [2][slots][rows][H] tagged fp32 words
  long long ag_off, flag_off;  // AG region [2][world * rows][H] bf16 + per-row flags [2][world * rows] u64
  int world, rank, rows, H, layers_per_step;
};
// Owner side of the reduce-scatter: res[t] += sum of the `slots` partials of token t; out[t] =
// rmsnorm(res[t]) * gamma; with ag_layer >= 0 the normed row is also all-gathered under that layer's tag.
void tp_rs_add_rmsnorm(const TpArgs& a, const int64_t* epoch, int layer, int slots, void* residual, const void* gamma,
                       void* out, long long ldo, float eps, int ag_layer, long long budget, int* err, int rows,
                       cudaStream_t s);
void tp_ag_send(const TpArgs& a, const int64_t* epoch, int layer, const void* x, long long ldx, int rows,
                cudaStream_t s);

// ---- block-scaled fp8 GEMM (gemm_fp8.cu)
// D[m, n] = sum_kb sa(m, kb) sb(n, kb) sum_{k in kb} A[m, k] B[n, k]; A, B e4m3 K-major,
// sa[(row / sa_rows) * ldsa + kb] (weight rows of A as stored), sb[kb * ldsb + n].
struct Fp8Launch {
  const void* A = nullptr;
  long long a_rows = 0, lda = 0;
  const float* sa = nullptr;
  long long ldsa = 0;
  int sa_rows = 128, sa_blocks = 0;  // scale rows: one per sa_rows weight rows
  const void* B = nullptr;
  long long b_rows = 0, ldb = 0;
  const float* sb = nullptr;
  long long ldsb = 0;
  void* D = nullptr;
  long long ldd = 0;
  int M = 0, N = 0, K = 0;
  int trans_out = 0, out_f32 = 0;
  int splits = 0, block_n = 0;
  int grouped = 0;
  const int* grp_rows = nullptr;
  const int* grp_tiles = nullptr;
  int num_groups = 0;
  int a_evict_first = 1;
  int swiglu = 0;
  float* ws = nullptr;
  long long ws_floats = 0;
  int slab_out = 0;
  int* err = nullptr;
  int num_sms = 148;
  cudaStream_t stream = 0;
  const EpComb* ep = nullptr;  // grouped only: send the output rows to their source ranks
};
int gemm_fp8(const Fp8Launch& g);
// Activation quantisation: row r (source row src_idx[r] / idx_div when src_idx is given) of
// bf16 x -> e4m3 q (pitch ldq) with one fp32 scale per 128 columns at s[kb * lds + r];
// rows_dev (optional) holds the live row count in device memory (rows = capacity).
void quant_act_fp8(const void* x, long long ldx, const int* src_idx, int idx_div, const int* rows_dev, void* q,
                   long long ldq, float* s, long long lds, int rows, int cols, int num_sms, cudaStream_t st);
// 128x128-block weight quantisation of bf16 `src` (or, when src is null, of seeded N(0, std)
// samples at flat indices flat0 + row * cols + col): q e4m3 [rows, cols], s [ceil(rows/128), cols/128].
void quant_weight_fp8(const void* src, uint64_t seed, long long flat0, float std_, void* q, float* s, int rows,
                      int cols, cudaStream_t st);

// ---- normalisation / rotary / KV cache (norm_rope.cu)
// residual (optional, in/out) += x; out = rmsnorm(residual or x) * w.
void add_rmsnorm(const void* x, long long ldx, void* residual, const void* w, void* out, long long ldo, int rows,
                 int hidden, float eps, cudaStream_t s);
// residual += sum of `splits` fp32 slabs ([rows, hidden] each, `stride` apart); out = rmsnorm(residual) * w
void slab_add_rmsnorm(const float* slab, long long stride, int splits, void* residual, const void* w, void* out,
                      long long ldo, int rows, int hidden, float eps, cudaStream_t s);
// Decode prologue of MLA attention from the q/kv projection row (bf16 `src` with pitch lds, or fp32 split-K
// slabs with row length row_len): cache <- [rmsnorm(latent), rope(k_pe)], q_nope_out [T, H, dn] <- q_nope,
// q_lat[t, h, kv_lora:] <- rope(q_pe).
void mla_decode_prep(const float* slab, long long stride, int splits, const void* src, long long lds,
                     const void* norm_w, const int* positions, const float* cos_sin, const int* slot_mapping,
                     void* cache, float* kv_scales, void* q_nope_out, void* q_lat, int T, int H, int dn, int dr,
                     int kv_lora, int q_off, int kv_off, int row_len, float eps, cudaStream_t s);
// kv: [T, kv_lora + rope] rows (pitch ldkv). Writes norm(latent)|rope(k_pe) into
// cache rows slot_mapping[t] (pitch kv_lora+rope) and, if latent_out != null,
// the same row into latent_out (pitch ldl).
void mla_kv_write(const void* kv, long long ldkv, const void* norm_w, const int* positions, const float* cos_sin,
                  const int* slot_mapping, void* cache, float* kv_scales, void* latent_out, long long ldl, int T,
                  int kv_lora, int rope, float eps, cudaStream_t s);
// With kv_scales set, `cache` is the fp8 cache [slots, 576] e4m3 and kv_scales its [slots, 5]
// fp32 block scales (amax / 448 per 128 elements; block 4 = the rope dims).
// In-place-capable RoPE on q: src[t, h, rope_off : rope_off+rope] -> dst[t, h, dst_off : dst_off+rope]
void rope_q(const void* src, long long src_tok, long long src_head, int src_off, void* dst, long long dst_tok,
            long long dst_head, int dst_off, const int* positions, const float* cos_sin, int T, int H, int rope,
            cudaStream_t s);
// fp8 e4m3 activation quantisation with one fp32 scale per 128-element block.
void quant_fp8_block(const void* x, long long ldx, void* q, float* scales, int rows, int cols, cudaStream_t s);

// ---- MLA decode attention (mla_decode.cu)
struct MlaDecodeLaunch {
  const void* q = nullptr;        // [B, H, kv_lora + rope] bf16
  const void* cache = nullptr;    // [num_slots, kv_lora + rope] bf16 (one layer)
  long long num_slots = 0;
  const int* block_table = nullptr;  // [B, max_blocks]
  int max_blocks = 0;
  const int* context_lens = nullptr; // [B]
  void* out = nullptr;            // [B, H, kv_lora] bf16
  float* o_part = nullptr;        // [B, splits, H, kv_lora] fp32 scratch
  float* lse_part = nullptr;      // [B, splits, H] fp32 scratch
  int B = 0, H = 0, kv_lora = 512, rope = 64, block_size = 64;
  int splits = 1;
  float scale = 1.f;
  int* err = nullptr;
  int impl = 0;                   // MLA_IMPL_*
  unsigned long long* trace = nullptr;  // tcgen05 kernel: [6][64] event times of CTA (0,0,0)
  int* counters = nullptr;        // stream-K kernel: per-row arrival counters, zero between launches
  int early = 0;                  // stream-K kernel: earlier-position KV may load before the PDL wait
  const int* last_slot = nullptr; // mma.sync kernel: [B] cache row of each row's last context token (-1: its block)
  const float* kv_scales = nullptr;  // fp8 cache: [num_slots, 5] block scales (cache is [num_slots, 576] e4m3)
  cudaStream_t stream = 0;
};
enum { MLA_IMPL_AUTO = 0, MLA_IMPL_TC = 1, MLA_IMPL_MMA = 2 };
// KV tokens per pipeline stage of the mma.sync decode kernel (64, or 32 when
// SPARKPIPE_MLA_STAGE_TOKENS=32) and how many decode CTAs of a head count fit on one SM.
int mla_stage_tokens();
int mla_ctas_per_sm(int heads, int impl = MLA_IMPL_AUTO);
void mla_decode(const MlaDecodeLaunch& l);
// fp8 (e4m3) cache with per-128 block scales (mla_decode_fp8.cu); same scratch and combine.
void mla_decode_fp8(const MlaDecodeLaunch& l);
int mla_fp8_ctas_per_sm(int heads);
// Split-KV merge of [B, splits, H, 512] partials and their log-sum-exps into out [B, H, 512] bf16.
void mla_combine(const float* o_part, const float* lse_part, void* out, int B, int H, int splits, cudaStream_t s);
// out[r, :] = dequantised fp8 cache row idx[r] (bf16 [n, 576]).
void kv8_gather(const void* cache8, const float* scales, const int* idx, void* out, int n, cudaStream_t s);
// Stream-K decode kernel (mla_decode_sk.cu): one CTA per SM over the flattened KV units.
// Scratch: o_part [segments][heads per CTA][512] fp32, lse_part [segments][heads per CTA],
// counters [(H / heads per CTA) * B] int32 zeroed once (the kernel leaves them zero).
bool mla_sk_supported(int B, int H);
int mla_sk_heads_per_cta(int heads);
long long mla_sk_segments(int B, int H, int num_sms);
void mla_decode_sk(const MlaDecodeLaunch& l, int num_sms);

// ---- DSA token selection (dsa.cu)
void paged_slots(const int* block_table, int max_blocks, const int* lens, const int* positions, int B, int rows,
                 int block_size, int* slots, cudaStream_t s);
void dsa_topk(const float* raw, const float* w, int B, int Hi, int rows, const int* lens, int topk, float* scores,
              int* out, int* counts, cudaStream_t s);

// ---- kernel resource receipts (registers, local memory, static shared memory) of
// the hot kernels, for the hardware probes; each file adds its own kernels.
struct KernelAttr {
  std::string name;
  int regs = 0, local_bytes = 0, static_smem = 0, max_threads = 0, ptx_version = 0, binary_version = 0;
};
template <class F>
inline void push_kernel_attr(std::vector<KernelAttr>& out, const std::string& name, F fn) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(fn)) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  out.push_back(KernelAttr{name, a.numRegs, (int)a.localSizeBytes, (int)a.sharedSizeBytes, a.maxThreadsPerBlock,
                           a.ptxVersion, a.binaryVersion});
}
void kernel_attrs_gemm(std::vector<KernelAttr>& out);
void kernel_attrs_fp8(std::vector<KernelAttr>& out);
void kernel_attrs_mla(std::vector<KernelAttr>& out);
void kernel_attrs_mla8(std::vector<KernelAttr>& out);
void kernel_attrs_mla_sk(std::vector<KernelAttr>& out);
void kernel_attrs_prefill(std::vector<KernelAttr>& out);
void kernel_attrs_moe(std::vector<KernelAttr>& out);

// ---- prefill attention (prefill_attn.cu)
struct PrefillAttnLaunch {
  const void* q = nullptr;  long long q_tok = 0, q_head = 0;      // [Tq, H, dn + dr]
  const void* k = nullptr;  long long k_tok = 0, k_head = 0;      // nope part [Tk, H, dn]
  const void* kpe = nullptr; long long kpe_tok = 0;               // rope part [Tk, dr] shared by heads
  const void* v = nullptr;  long long v_tok = 0, v_head = 0;      // [Tk, H, dv]
  void* o = nullptr;        long long o_tok = 0, o_head = 0;      // [Tq, H, dv]
  const int* cu_q = nullptr; const int* cu_k = nullptr;           // [B + 1]
  int B = 0, H = 0, max_q = 0;
  int dn = 128, dr = 64, dv = 128;
  float scale = 1.f;
  int causal = 1;
  long long q_rows = 0, k_rows = 0;  // rows of the q / k (kpe, v) tensors (TMA extents)
  int impl = 0;                       // ATTN_IMPL_*
  int* err = nullptr;
  cudaStream_t stream = 0;
};
enum { ATTN_IMPL_AUTO = 0, ATTN_IMPL_TC = 1, ATTN_IMPL_MMA = 2 };
void prefill_attention(const PrefillAttnLaunch& l);
bool prefill_attention_tc_ok(const PrefillAttnLaunch& l);
void prefill_attention_tc(const PrefillAttnLaunch& l);

// ---- MoE routing (moe.cu)
// scoring: 0 = softmax, 1 = sigmoid (+bias for selection). Weights are renormalised
// over the selected experts when renorm != 0, then multiplied by `scaling`.
// The last n_shared columns of topk_ids / topk_w are the shared experts E .. E+n_shared-1 (weight 1).
// `logits` may be split-K slabs: the logits are sum_s logits[s * slab_stride + ...] over `splits`.
void moe_topk(const float* logits, long long slab_stride, int splits, const float* bias, int* topk_ids, float* topk_w,
              int T, int E, int k, int n_shared, int scoring, int renorm, float scaling, int n_group, int topk_group,
              int group_top2, cudaStream_t s, const void* gate_x = nullptr, long long ldx = 0,
              const void* gate_w = nullptr, int H = 0);
// res[t] += sum_j w[t, j] * y[inv_pos[t*k + j]]; out[t] = rmsnorm(res[t]) * gamma
void combine_add_rmsnorm(const void* y, long long ldy, const int* inv_pos, const float* topk_w, void* residual,
                         const void* gamma, void* out, long long ldo, int T, int k, int H, float eps, cudaStream_t s,
                         const void* shared = nullptr, long long ld_shared = 0, int n_shared = 0);
// Builds the expert-sorted row layout: counts -> grp_rows [E+1], grp_tiles [E+1]
// (n-tiles of width block_n), sorted_tok [T*k] (source token of each sorted row),
// inv_pos [T*k] (sorted row of pair (t, j)). `work` is E ints of scratch.
// Returns the number of kernels launched.
int moe_align(const int* topk_ids, int T, int k, int E, int block_n, int* grp_rows, int* grp_tiles,
               int* sorted_tok, int* inv_pos, int* work, cudaStream_t s);
void gather_rows(const void* x, long long ldx, const int* idx, void* out, long long ldo, int rows, int cols,
                 cudaStream_t s);
void silu_mul(const void* h, long long ldh, void* out, long long ldo, int rows, int F, cudaStream_t s);
// out[t] = sum_j w[t, j] * y[inv_pos[t*k + j]] (+ add[t] if add != null)
void moe_combine(const void* y, long long ldy, const int* inv_pos, const float* topk_w, const void* add,
                 long long ld_add, void* out, long long ldo, int T, int k, int H, cudaStream_t s);

// ---- sampling / embedding / speculative verify (sampling.cu)
void embedding(const void* table, long long ld, const int* ids, void* out, long long ldo, int T, int H,
               cudaStream_t s);
// temperature <= 0 -> greedy argmax; else Gumbel-max sampling seeded by (seed, offset, row).
void sample_tokens(const void* logits, long long ldl, int T, int V, float temperature, unsigned long long seed,
                   unsigned long long offset, int* out_ids, float* out_logit, const float* row_temp,
                   const unsigned long long* row_key, cudaStream_t s);
void gather_prev_tokens(int* ids, const int* prev, int n, int prev_rows, cudaStream_t s);
// NVFP4 (E2M1 values, E4M3 scale per 16, FP32 tensor scale) rows to bf16
void dequant_nvfp4(const uint8_t* packed, const uint8_t* scales, float tensor_scale, long long elements, void* out,
                   cudaStream_t s);
// Greedy speculative verification over a chain of L drafts per row.
// target: [B, L+1] argmax tokens of the verifier; draft: [B, L].
// forced_accept_p > 0 replaces the token comparison by a seeded Bernoulli(p).
void spec_verify(const int* draft, const int* target, int B, int L, float forced_accept_p, unsigned long long seed,
                 unsigned long long offset, int* accepted, int* committed, cudaStream_t s);

// End of a speculative round over j-major row arrays (row j*B + b, j = 0..L): acceptance, committed
// tokens, and the next round's inputs (see sampling.cu).
// Verify kernels of the serving engine (spec_verify.cu); row arrays [rows][B].
void spec_chain_commit(const int* tok, const int* tgt, const int* ctx, const int* pos, const int* budget,
                       const unsigned long long* keys, int B, int L, float p_accept, unsigned long long seed,
                       int* committed, int* counts, cudaStream_t s);
void mtp_tree_commit(const int* tok, const int* tgt, const int* ctx, const int* slots, int B, void* cache,
                     long long layer_stride, int layers, int row_elems, int* committed, int* counts, int* paths,
                     cudaStream_t s, float* aux = nullptr, long long aux_layer_stride = 0, int aux_row = 0);
void top2_rows(const void* logits, long long ldl, int T, int V, int* out0, int* out1, cudaStream_t s);
void spec_finish(int* tok_rows, const int* tgt_rows, int B, int L, float p_accept, unsigned long long seed,
                 int* pos_rows, int* ctx_rows, int* slot_rows, const int* block_table, int max_blocks,
                 int block_size, int* accepted, int* committed, unsigned long long* total_committed, cudaStream_t s);
// Paged KV blocks of a [layers][slots][row] bf16 cache <-> staging [n][layers][block_size][row].
void kv_blocks_copy(void* cache, long long layer_stride, const int* blocks, int n, void* staging, int layers,
                    int block_size, int row, int to_staging, cudaStream_t s);
// Phase clocks: totals[slot] += now - stamps[prev] (prev >= 0); stamps[slot] <- device global timer (ns).
void phase_mark(unsigned long long* stamps, unsigned long long* totals, int slot, int prev, cudaStream_t s);
void decode_advance(const int* out_ids, int* ids, int* pos, int* ctx, int* slots, const int* block_table,
                    int max_blocks, int B, int block_size, cudaStream_t s);

// ---- expert-parallel dispatch / combine over peer memory (ep.cu)
constexpr int EP_MAX_RANKS = 8;
constexpr int EP_MAX_KK = 16;
constexpr int EP_CHUNK_TOKENS = 8;   // tokens per dispatch CTA (at most 32)
constexpr int EP_COMBINE_CTAS = 16;  // combine-send CTAs per destination
// Every rank's EP buffer (mapped into this process) plus the byte offsets of
// its regions; identical on all ranks except `rank`.
struct EpArgs {
  unsigned long long base[EP_MAX_RANKS];
  long long off_ctrl, off_nch, off_meta, off_rows, off_comb;
  int world, rank, cap, H, kk, n_routed, experts_per_rank, n_shared, moe_layers, max_chunks;
  int fp8;              // dispatched rows travel as e4m3 + one fp32 scale per 128 columns
  long long row_words;  // tagged words per dispatched row (H/2 bf16; H/4 + even(H/128) fp8)
  int shared_local;     // shared experts (ids >= n_routed) are not dispatched: each rank runs them on
                        // its own tokens while the routed rows travel, and the combine reads their rows
};
constexpr int EP_ARGS_WORDS = EP_MAX_RANKS + 5 + 10 + 3;
void ep_dispatch(const void* x, int64_t ldx, const int* ids, int T, const EpArgs& a, const int64_t* epoch, int layer,
                 cudaStream_t s);
void ep_recv_align(const EpArgs& a, const int64_t* epoch, int layer, int bn, int* grp_rows, int* grp_tiles,
                   int* src_row, int* comb_dst, long long budget, int* err, cudaStream_t s);
// fp8 transport: received rows -> expert-sorted e4m3 rows xq [*, H] (pitch ldq) and
// K-block-major scales xs_scale[kb * lds + row]
void ep_gather_fp8(const EpArgs& a, const int64_t* epoch, int layer, const int* total, const int* src_row, void* xq,
                   long long ldq, float* xs_scale, long long lds, long long budget, int* err, int num_sms,
                   cudaStream_t s);
void ep_gather(const EpArgs& a, const int64_t* epoch, int layer, const int* total, const int* src_row, void* xs,
               long long budget, int* err, int num_sms, cudaStream_t s);
void ep_combine_send(const void* y, const int* total, const int* comb_dst, const EpArgs& a, const int64_t* epoch,
                     int layer, cudaStream_t s);
// y_shared (shared_local): [n_shared, T, H] bf16 outputs of the shared experts, slots kk - n_shared .. kk - 1.
void ep_combine_add_rmsnorm(const EpArgs& a, const int64_t* epoch, int layer, const float* topk_w, void* residual,
                            const void* gamma, void* out, long long ldo, int T, float eps, long long budget, int* err,
                            const void* y_shared, cudaStream_t s);
void ep_advance(int64_t* epoch, cudaStream_t s);

}  // namespace sp
