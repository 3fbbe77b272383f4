// torch bindings of the sm_100a kernels. Every op launches on the current CUDA
// stream (so it can be captured into a CUDA graph) and checks the device, dtype
// and contiguity assumptions of its kernel before launching.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "launch.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be fp32")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
// every operand a kernel dereferences lives on the launching tensor's device
#define CHECK_ON(ref, x) \
  TORCH_CHECK((x).is_cuda() && (x).device() == (ref).device(), #x " must be a CUDA tensor on " #ref "'s device")

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// Per-device status word written by kernels on a bounded-wait timeout.
std::mutex g_mu;
std::unordered_map<int, int*> g_err;
std::unordered_map<int, int> g_sms;

// Per-device split-K workspace: the fp32 partial slabs of one split GEMM. Split
// GEMMs on a device must be stream-ordered (PDL keeps that order: a kernel
// writes its slabs only after its predecessor has finished).
constexpr long long kSplitWsFloats = 8ll << 20;  // 32 MiB
std::unordered_map<int, float*> g_split;

float* split_ws() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_split.find(dev);
  if (it != g_split.end()) return it->second;
  float* w = nullptr;
  TORCH_CHECK(cudaMalloc(&w, sizeof(float) * kSplitWsFloats) == cudaSuccess, "split-K workspace allocation");
  g_split[dev] = w;
  return w;
}

int* err_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_err.find(dev);
  if (it != g_err.end()) return it->second;
  int* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, sizeof(int)) == cudaSuccess, "cannot allocate the kernel status word");
  TORCH_CHECK(cudaMemset(p, 0, sizeof(int)) == cudaSuccess, "cannot clear the kernel status word");
  g_err[dev] = p;
  return p;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sms.find(dev);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  g_sms[dev] = n;
  return n;
}

int status_word() {
  int* p = err_word();
  int v = 0;
  TORCH_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess, "status read failed");
  return v;
}

void clear_status() {
  int* p = err_word();
  TORCH_CHECK(cudaMemset(p, 0, sizeof(int)) == cudaSuccess, "status clear failed");
}

sp::EpArgs ep_args(const std::vector<int64_t>& v);

// Expert-parallel combine epilogue of a grouped GEMM: (EP argument vector, comb_dst, epoch, MoE layer).
bool fill_ep_comb(sp::EpComb& e, const std::vector<int64_t>& ep, const c10::optional<Tensor>& comb_dst,
                  const c10::optional<Tensor>& epoch, int64_t layer) {
  if (ep.empty()) return false;
  TORCH_CHECK(comb_dst.has_value() && epoch.has_value(), "ep combine epilogue: comb_dst and epoch are required");
  CHECK_I32(*comb_dst);
  TORCH_CHECK(epoch->scalar_type() == at::kLong, "ep combine epilogue: epoch must be int64");
  const sp::EpArgs a = ep_args(ep);
  for (int r = 0; r < 8; ++r) e.base[r] = a.base[r];
  e.comb_off = a.off_comb; e.cap = a.cap; e.kk = a.kk; e.H = a.H; e.layers_per_step = a.moe_layers;
  e.comb_dst = comb_dst->data_ptr<int>();
  e.epoch = epoch->data_ptr<int64_t>();
  e.layer = (int)layer;
  return true;
}

int64_t gemm(const Tensor& A, const Tensor& B, const Tensor& D, int64_t a_rows, int64_t a_cols, int64_t lda,
          int64_t b_rows, int64_t b_cols, int64_t ldb, int64_t ldd, int64_t d_batch_stride, int64_t M, int64_t N,
          int64_t K, int64_t batch, int64_t a_row0, int64_t a_batch_rows, int64_t a_k0, int64_t a_batch_k,
          int64_t b_row0, int64_t b_batch_rows, int64_t b_k0, int64_t b_batch_k, int64_t trans_out, int64_t splits,
          int64_t block_n, const c10::optional<Tensor>& grp_rows, const c10::optional<Tensor>& grp_tiles,
          int64_t num_groups, int64_t a_evict_first, int64_t swiglu, int64_t slab_out,
          const std::vector<int64_t>& ep, const c10::optional<Tensor>& comb_dst, const c10::optional<Tensor>& epoch,
          int64_t ep_layer, int64_t sched_early) {
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(D);
  CHECK_BF16(A); CHECK_BF16(B);
  TORCH_CHECK(D.scalar_type() == at::kBFloat16 || D.scalar_type() == at::kFloat, "D must be bf16 or fp32");
  const c10::cuda::CUDAGuard guard(A.device());
  sp::GemmLaunch g;
  g.A = A.data_ptr(); g.a_rows = a_rows; g.a_cols = a_cols; g.lda = lda;
  g.B = B.data_ptr(); g.b_rows = b_rows; g.b_cols = b_cols; g.ldb = ldb;
  g.D = D.data_ptr(); g.ldd = ldd; g.d_batch_stride = d_batch_stride;
  g.M = (int)M; g.N = (int)N; g.K = (int)K; g.batch = (int)batch;
  g.a_row0 = (int)a_row0; g.a_batch_rows = (int)a_batch_rows; g.a_k0 = (int)a_k0; g.a_batch_k = (int)a_batch_k;
  g.b_row0 = (int)b_row0; g.b_batch_rows = (int)b_batch_rows; g.b_k0 = (int)b_k0; g.b_batch_k = (int)b_batch_k;
  g.trans_out = (int)trans_out;
  g.out_f32 = D.scalar_type() == at::kFloat ? 1 : 0;
  g.splits = (int)splits;
  g.block_n = (int)block_n;
  if (grp_rows.has_value()) {
    TORCH_CHECK(grp_tiles.has_value(), "grouped GEMM needs grp_tiles");
    CHECK_I32(*grp_rows); CHECK_I32(*grp_tiles);
    g.grouped = 1;
    g.grp_rows = grp_rows->data_ptr<int>();
    g.grp_tiles = grp_tiles->data_ptr<int>();
    g.num_groups = (int)num_groups;
  }
  g.a_evict_first = (int)a_evict_first;
  g.sched_early = (int)sched_early;
  g.swiglu = (int)swiglu;
  if (!grp_rows.has_value() && splits != 1) {
    g.ws = split_ws();
    g.ws_floats = kSplitWsFloats;
  }
  g.slab_out = (int)slab_out;
  g.err = err_word();
  g.num_sms = num_sms();
  g.stream = stream();
  sp::EpComb ec;
  if (fill_ep_comb(ec, ep, comb_dst, epoch, ep_layer)) g.ep = &ec;
  return sp::gemm_bf16(g);
}

// Token-major grouped expert GEMM for prefill-size groups: out[r] = W[g(r)] x[r] for
// rows sorted by group (grp_tiles counts 128-row token tiles), W as [groups x n, K];
// with swiglu (W interleaved [64 gate | 64 up] per 128 rows) out[r] = silu(gate) * up.
int64_t grouped_gemm_tm(const Tensor& x, const Tensor& w, const Tensor& out, const Tensor& grp_rows,
                        const Tensor& grp_tiles, int64_t num_groups, int64_t n, int64_t block_n, int64_t swiglu) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(out); CHECK_I32(grp_rows); CHECK_I32(grp_tiles);
  CHECK_ON(x, w); CHECK_ON(x, out); CHECK_ON(x, grp_rows); CHECK_ON(x, grp_tiles);
  CHECK_CONTIG(x); CHECK_CONTIG(w); CHECK_CONTIG(out);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "grouped_gemm_tm: 2-D operands");
  const int64_t K = x.size(1);
  TORCH_CHECK(w.size(1) == K && w.size(0) == num_groups * n, "grouped_gemm_tm: W is [groups x n, K]");
  TORCH_CHECK(out.size(0) >= x.size(0) && out.size(1) >= (swiglu ? n / 2 : n), "grouped_gemm_tm: output too small");
  TORCH_CHECK(grp_rows.numel() > num_groups && grp_tiles.numel() > num_groups, "grouped_gemm_tm: group tables");
  const c10::cuda::CUDAGuard guard(x.device());
  sp::GemmLaunch g;
  g.A = x.data_ptr(); g.a_rows = x.size(0); g.a_cols = K; g.lda = x.stride(0);
  g.B = w.data_ptr(); g.b_rows = w.size(0); g.b_cols = K; g.ldb = w.stride(0);
  g.D = out.data_ptr(); g.ldd = out.stride(0);
  g.M = (int)x.size(0); g.N = (int)n; g.K = (int)K;
  g.b_batch_rows = (int)n;
  g.grouped = 2;
  g.grp_rows = grp_rows.data_ptr<int>();
  g.grp_tiles = grp_tiles.data_ptr<int>();
  g.num_groups = (int)num_groups;
  g.block_n = (int)block_n;
  g.swiglu = (int)swiglu;
  g.err = err_word();
  g.num_sms = num_sms();
  g.stream = stream();
  return sp::gemm_bf16(g);
}

// ---- tensor parallelism (tp.cu, gemm_tcgen05.cu)
constexpr int kTpArgsWords = 8 + 3 + 5;

sp::TpArgs tp_args(const std::vector<int64_t>& v) {
  TORCH_CHECK((int)v.size() == kTpArgsWords, "tp: argument vector must hold ", kTpArgsWords, " words");
  sp::TpArgs a{};
  int i = 0;
  for (int r = 0; r < 8; ++r) a.base[r] = (unsigned long long)v[i++];
  a.rs_off = v[i++]; a.ag_off = v[i++]; a.flag_off = v[i++];
  a.world = (int)v[i++]; a.rank = (int)v[i++]; a.rows = (int)v[i++]; a.H = (int)v[i++];
  a.layers_per_step = (int)v[i++];
  return a;
}

int64_t gemm_tp(const Tensor& A, const c10::optional<Tensor>& B, const Tensor& D, int64_t M, int64_t N, int64_t K,
                const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, int64_t rs, int64_t ag,
                int64_t rs_M, int64_t splits, int64_t block_n, int64_t budget_cycles) {
  // rs: D is unused (partials go to the owners' reduce-scatter slots, rs_M = features per token);
  // ag: B is unused (rows come from this rank's all-gather region, row length = args' H)
  CHECK_CUDA(A); CHECK_BF16(A); CHECK_CUDA(D);
  TORCH_CHECK(A.dim() == 2 && A.stride(1) == 1, "gemm_tp: A must be a 2-D row-major view");
  TORCH_CHECK(epoch.scalar_type() == at::kLong && epoch.is_cuda(), "gemm_tp: epoch must be a CUDA int64 tensor");
  const c10::cuda::CUDAGuard guard(A.device());
  const sp::TpArgs a = tp_args(args);
  sp::TpGemm t;
  for (int r = 0; r < 8; ++r) t.base[r] = a.base[r];
  t.rs_off = a.rs_off; t.rs = rs ? 1 : 0; t.rank = a.rank; t.world = a.world; t.rows = a.rows;
  t.epoch = epoch.data_ptr<int64_t>(); t.layer = (int)layer; t.layers_per_step = a.layers_per_step;
  t.budget = budget_cycles;
  sp::GemmLaunch g;
  g.A = A.data_ptr(); g.a_rows = A.size(0); g.a_cols = A.size(1); g.lda = A.stride(0);
  if (ag) {
    t.ag_flags = reinterpret_cast<const void*>(a.base[a.rank] + a.flag_off);
    g.B = reinterpret_cast<const void*>(a.base[a.rank] + a.ag_off);  // [2 x world x rows, H] bf16
    g.b_rows = 2ll * a.world * a.rows; g.b_cols = a.H; g.ldb = a.H;
  } else {
    TORCH_CHECK(B.has_value(), "gemm_tp: B is required without the all-gather operand");
    CHECK_BF16(*B);
    TORCH_CHECK(B->dim() == 2 && B->stride(1) == 1, "gemm_tp: B must be a 2-D row-major view");
    g.B = B->data_ptr(); g.b_rows = B->size(0); g.b_cols = B->size(1); g.ldb = B->stride(0);
  }
  if (rs) {
    TORCH_CHECK(rs_M == M, "gemm_tp: reduce-scatter features must equal M");
  } else {
    TORCH_CHECK(D.scalar_type() == at::kBFloat16 || D.scalar_type() == at::kFloat, "D must be bf16 or fp32");
  }
  g.D = D.data_ptr(); g.ldd = D.dim() == 2 ? D.stride(0) : M;
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.trans_out = 1;
  g.out_f32 = D.scalar_type() == at::kFloat ? 1 : 0;
  g.splits = rs ? (int)splits : 1;
  g.block_n = (int)block_n;
  g.a_evict_first = 1;
  g.err = err_word();
  g.num_sms = num_sms();
  g.stream = stream();
  g.tp = &t;
  return sp::gemm_bf16(g);
}

void tp_rs_add_rmsnorm(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, int64_t slots,
                       const Tensor& residual, const Tensor& gamma, const Tensor& out, double eps, int64_t ag_layer,
                       int64_t budget_cycles) {
  CHECK_CUDA(residual); CHECK_BF16(residual); CHECK_BF16(gamma); CHECK_BF16(out); CHECK_CONTIG(residual);
  TORCH_CHECK(out.stride(1) == 1 && out.stride(0) % 8 == 0, "tp: out rows must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(residual.device());
  const sp::TpArgs a = tp_args(args);
  TORCH_CHECK(residual.size(1) == a.H && out.size(0) >= residual.size(0), "tp: shapes");
  sp::tp_rs_add_rmsnorm(a, epoch.data_ptr<int64_t>(), (int)layer, (int)slots, residual.data_ptr(), gamma.data_ptr(),
                        out.data_ptr(), out.stride(0), (float)eps, (int)ag_layer, budget_cycles, err_word(),
                        (int)residual.size(0), stream());
}

void tp_ag_send(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, const Tensor& x) {
  CHECK_CUDA(x); CHECK_BF16(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "tp: x rows must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(x.device());
  const sp::TpArgs a = tp_args(args);
  TORCH_CHECK(x.size(1) == a.H, "tp: x width");
  sp::tp_ag_send(a, epoch.data_ptr<int64_t>(), (int)layer, x.data_ptr(), x.stride(0), (int)x.size(0), stream());
}

void add_rmsnorm(const Tensor& x, const c10::optional<Tensor>& residual, const Tensor& w, const Tensor& out,
                 double eps) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(out);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "add_rmsnorm: 2-D row-major");
  const c10::cuda::CUDAGuard guard(x.device());
  void* r = nullptr;
  if (residual.has_value()) {
    CHECK_BF16(*residual); CHECK_CONTIG(*residual);
    r = residual->data_ptr();
  }
  sp::add_rmsnorm(x.data_ptr(), x.stride(0), r, w.data_ptr(), out.data_ptr(), out.stride(0), (int)x.size(0),
                  (int)x.size(1), (float)eps, stream());
}

// The latent KV cache is bf16 [.., slots, 576], or e4m3 [.., slots, 576] (uint8 or float8_e4m3fn)
// with its fp32 block scales [.., slots, 5]; returns the scales pointer (null for bf16).
static float* kv8_scales(const Tensor& cache, const c10::optional<Tensor>& scales, const char* who) {
  const bool fp8 = cache.scalar_type() == at::kByte || cache.scalar_type() == at::kFloat8_e4m3fn;
  if (!fp8) {
    TORCH_CHECK(cache.scalar_type() == at::kBFloat16, who, ": cache must be bf16 or fp8 e4m3");
    TORCH_CHECK(!scales.has_value(), who, ": scales given for a bf16 cache");
    return nullptr;
  }
  TORCH_CHECK(scales.has_value(), who, ": an fp8 cache needs its block scales");
  TORCH_CHECK(scales->scalar_type() == at::kFloat && scales->is_contiguous() && scales->size(-1) == 5,
              who, ": scales must be contiguous fp32 [.., slots, 5]");
  TORCH_CHECK(cache.size(-1) == 576 && cache.is_contiguous(), who, ": fp8 cache rows of 576, contiguous");
  TORCH_CHECK(scales->numel() / 5 == cache.numel() / 576, who, ": one scale row per cache row");
  TORCH_CHECK(scales->device() == cache.device(), who, ": scales on another device");
  return scales->data_ptr<float>();
}

void mla_kv_write(const Tensor& kv, const Tensor& norm_w, const Tensor& positions, const Tensor& cos_sin,
                  const c10::optional<Tensor>& slot_mapping, const Tensor& cache,
                  const c10::optional<Tensor>& latent_out, int64_t kv_lora, int64_t rope, double eps,
                  const c10::optional<Tensor>& kv_scales) {
  CHECK_CUDA(kv); CHECK_BF16(kv); CHECK_BF16(norm_w); CHECK_I32(positions); CHECK_F32(cos_sin);
  float* ks = kv8_scales(cache, kv_scales, "mla_kv_write");
  TORCH_CHECK(kv.stride(1) == 1, "kv rows must be contiguous");
  const c10::cuda::CUDAGuard guard(kv.device());
  const int* slots = nullptr;
  if (slot_mapping.has_value()) { CHECK_I32(*slot_mapping); slots = slot_mapping->data_ptr<int>(); }
  void* lat = nullptr;
  long long ldl = 0;
  if (latent_out.has_value()) { CHECK_BF16(*latent_out); lat = latent_out->data_ptr(); ldl = latent_out->stride(0); }
  sp::mla_kv_write(kv.data_ptr(), kv.stride(0), norm_w.data_ptr(), positions.data_ptr<int>(),
                   cos_sin.data_ptr<float>(), slots, cache.data_ptr(), ks, lat, ldl, (int)kv.size(0), (int)kv_lora,
                   (int)rope, (float)eps, stream());
}

void rope_q(const Tensor& src, int64_t src_off, const Tensor& dst, int64_t dst_off, const Tensor& positions,
            const Tensor& cos_sin, int64_t rope) {
  // src/dst: [T, H, *] with unit innermost stride
  CHECK_CUDA(src); CHECK_BF16(src); CHECK_BF16(dst); CHECK_I32(positions); CHECK_F32(cos_sin);
  TORCH_CHECK(src.dim() == 3 && dst.dim() == 3 && src.stride(2) == 1 && dst.stride(2) == 1, "rope_q: [T, H, D]");
  const c10::cuda::CUDAGuard guard(src.device());
  sp::rope_q(src.data_ptr(), src.stride(0), src.stride(1), (int)src_off, dst.data_ptr(), dst.stride(0),
             dst.stride(1), (int)dst_off, positions.data_ptr<int>(), cos_sin.data_ptr<float>(), (int)src.size(0),
             (int)src.size(1), (int)rope, stream());
}

void quant_fp8_block(const Tensor& x, const Tensor& q, const Tensor& scales) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_F32(scales);
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn, "q must be float8_e4m3fn");
  CHECK_CONTIG(q); CHECK_CONTIG(scales);
  const c10::cuda::CUDAGuard guard(x.device());
  sp::quant_fp8_block(x.data_ptr(), x.stride(0), q.data_ptr(), scales.data_ptr<float>(), (int)x.size(0),
                      (int)x.size(1), stream());
}

#define CHECK_FP8(x) \
  TORCH_CHECK((x).scalar_type() == at::kFloat8_e4m3fn || (x).scalar_type() == at::kByte, #x " must be e4m3 (or bytes)")

int64_t gemm_fp8(const Tensor& A, const Tensor& sa, int64_t sa_rows, const Tensor& B, const Tensor& sb,
                 const Tensor& D, int64_t M, int64_t N, int64_t K, int64_t trans_out, int64_t splits, int64_t block_n,
                 const c10::optional<Tensor>& grp_rows, const c10::optional<Tensor>& grp_tiles, int64_t num_groups,
                 int64_t swiglu, int64_t slab_out, const std::vector<int64_t>& ep,
                 const c10::optional<Tensor>& comb_dst, const c10::optional<Tensor>& epoch, int64_t ep_layer) {
  // A: weights [rows, K] e4m3 (2-D row-major view), sa [rows / sa_rows, K / 128] fp32;
  // B: activations [b_rows, K] e4m3, sb [K / 128, ldsb] fp32 (K-block-major)
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(D); CHECK_FP8(A); CHECK_FP8(B); CHECK_F32(sa); CHECK_F32(sb);
  TORCH_CHECK(A.dim() == 2 && A.stride(1) == 1 && B.dim() == 2 && B.stride(1) == 1, "gemm_fp8: 2-D row-major operands");
  TORCH_CHECK(sa.dim() == 2 && sa.stride(1) == 1 && sb.dim() == 2 && sb.stride(1) == 1, "gemm_fp8: 2-D scale views");
  TORCH_CHECK(sb.size(0) * 128 >= K && sa.size(1) * 128 >= K, "gemm_fp8: scale columns do not cover K");
  TORCH_CHECK(sa.size(0) * sa_rows >= A.size(0), "gemm_fp8: weight scales do not cover A's rows");
  TORCH_CHECK(D.scalar_type() == at::kBFloat16 || D.scalar_type() == at::kFloat, "D must be bf16 or fp32");
  const c10::cuda::CUDAGuard guard(A.device());
  sp::Fp8Launch g;
  g.A = A.data_ptr(); g.a_rows = A.size(0); g.lda = A.stride(0);
  g.sa = sa.data_ptr<float>(); g.ldsa = sa.stride(0); g.sa_rows = (int)sa_rows; g.sa_blocks = (int)sa.size(0);
  g.B = B.data_ptr(); g.b_rows = B.size(0); g.ldb = B.stride(0);
  g.sb = sb.data_ptr<float>(); g.ldsb = sb.stride(0);
  TORCH_CHECK(g.ldsb >= B.size(0), "gemm_fp8: activation scale pitch shorter than B's rows");
  g.D = D.data_ptr(); g.ldd = D.stride(0);
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.trans_out = (int)trans_out;
  g.out_f32 = D.scalar_type() == at::kFloat ? 1 : 0;
  g.splits = (int)splits;
  g.block_n = (int)block_n;
  if (grp_rows.has_value()) {
    TORCH_CHECK(grp_tiles.has_value(), "grouped GEMM needs grp_tiles");
    CHECK_I32(*grp_rows); CHECK_I32(*grp_tiles);
    g.grouped = 1;
    g.grp_rows = grp_rows->data_ptr<int>();
    g.grp_tiles = grp_tiles->data_ptr<int>();
    g.num_groups = (int)num_groups;
    TORCH_CHECK(A.size(0) >= (int64_t)num_groups * M, "gemm_fp8: A holds fewer than num_groups x M rows");
  } else {
    TORCH_CHECK(A.size(0) >= M && B.size(0) >= N, "gemm_fp8: operands smaller than M / N");
    if (splits != 1) {
      g.ws = split_ws();
      g.ws_floats = kSplitWsFloats;
    }
  }
  g.a_evict_first = 1;
  g.swiglu = (int)swiglu;
  g.slab_out = (int)slab_out;
  g.err = err_word();
  g.num_sms = num_sms();
  g.stream = stream();
  sp::EpComb ec;
  if (fill_ep_comb(ec, ep, comb_dst, epoch, ep_layer)) g.ep = &ec;
  return sp::gemm_fp8(g);
}

void quant_act_fp8(const Tensor& x, const c10::optional<Tensor>& src_idx, int64_t idx_div,
                   const c10::optional<Tensor>& rows_dev, const Tensor& q, const Tensor& s) {
  // q [rows, K] e4m3; s [K / 128, lds] fp32; rows = q.size(0) (gathered from x when src_idx is given)
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_FP8(q); CHECK_F32(s);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && q.dim() == 2 && q.stride(1) == 1 && s.dim() == 2 &&
                  s.stride(1) == 1, "quant_act_fp8: 2-D row-major views");
  const int64_t rows = q.size(0), cols = q.size(1);
  TORCH_CHECK(x.size(1) == cols && s.size(0) * 128 == cols && s.stride(0) >= rows, "quant_act_fp8: shapes");
  const int* idx = nullptr;
  if (src_idx.has_value()) {
    CHECK_I32(*src_idx);
    TORCH_CHECK(src_idx->numel() >= rows, "quant_act_fp8: gather index shorter than the rows");
    idx = src_idx->data_ptr<int>();
  } else {
    TORCH_CHECK(x.size(0) >= rows, "quant_act_fp8: x has fewer rows than q");
  }
  const int* rd = nullptr;
  if (rows_dev.has_value()) {
    CHECK_I32(*rows_dev);
    rd = rows_dev->data_ptr<int>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  sp::quant_act_fp8(x.data_ptr(), x.stride(0), idx, (int)idx_div, rd, q.data_ptr(), q.stride(0),
                    s.data_ptr<float>(), s.stride(0), (int)rows, (int)cols, num_sms(), stream());
}

void quant_weight_fp8(const c10::optional<Tensor>& src, int64_t seed, int64_t flat0, double std_, const Tensor& q,
                      const Tensor& s) {
  // q [rows, cols] e4m3 contiguous; s [ceil(rows / 128), cols / 128] fp32 contiguous
  CHECK_CUDA(q); CHECK_FP8(q); CHECK_F32(s); CHECK_CONTIG(q); CHECK_CONTIG(s);
  TORCH_CHECK(q.dim() == 2, "quant_weight_fp8: 2-D weight");
  const int64_t rows = q.size(0), cols = q.size(1);
  TORCH_CHECK(s.numel() == ((rows + 127) / 128) * (cols / 128), "quant_weight_fp8: scale shape");
  const void* sp_ = nullptr;
  if (src.has_value()) {
    CHECK_BF16(*src); CHECK_CONTIG(*src);
    TORCH_CHECK(src->numel() == rows * cols, "quant_weight_fp8: source shape");
    sp_ = src->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(q.device());
  sp::quant_weight_fp8(sp_, (uint64_t)seed, flat0, (float)std_, q.data_ptr(), s.data_ptr<float>(), (int)rows,
                       (int)cols, stream());
}

void mla_decode(const Tensor& q, const Tensor& cache, const Tensor& block_table, const Tensor& context_lens,
                const Tensor& out, const c10::optional<Tensor>& o_part, const c10::optional<Tensor>& lse_part,
                int64_t splits, double scale, int64_t impl, const c10::optional<Tensor>& trace,
                const c10::optional<Tensor>& last_slot, const c10::optional<Tensor>& kv_scales) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_I32(block_table); CHECK_I32(context_lens); CHECK_BF16(out);
  const float* ks = kv8_scales(cache, kv_scales, "mla_decode");
  CHECK_ON(q, cache); CHECK_ON(q, block_table); CHECK_ON(q, context_lens); CHECK_ON(q, out);
  CHECK_CONTIG(q); CHECK_CONTIG(block_table); CHECK_CONTIG(out);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 576, "q: [B, H, 576]");
  TORCH_CHECK(cache.size(-1) == 576 && cache.stride(-1) == 1, "cache rows of 576");
  const c10::cuda::CUDAGuard guard(q.device());
  sp::MlaDecodeLaunch l;
  l.q = q.data_ptr();
  l.cache = cache.data_ptr();
  l.num_slots = cache.numel() / 576;
  l.block_table = block_table.data_ptr<int>();
  l.max_blocks = (int)block_table.size(1);
  l.context_lens = context_lens.data_ptr<int>();
  l.out = out.data_ptr();
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(block_table.size(0) >= B && context_lens.numel() >= B, "mla_decode: block table / lengths too short");
  TORCH_CHECK(out.numel() >= B * H * 512, "mla_decode: output too small");
  if (o_part.has_value()) {
    CHECK_F32(*o_part); CHECK_ON(q, *o_part);
    TORCH_CHECK(o_part->numel() >= B * splits * H * 512, "mla_decode: split partials too small");
    l.o_part = o_part->data_ptr<float>();
  }
  if (lse_part.has_value()) {
    CHECK_F32(*lse_part); CHECK_ON(q, *lse_part);
    TORCH_CHECK(lse_part->numel() >= B * splits * H, "mla_decode: split log-sum-exps too small");
    l.lse_part = lse_part->data_ptr<float>();
  }
  l.B = (int)B;
  l.H = (int)H;
  l.splits = (int)splits;
  l.impl = (int)impl;
  if (trace.has_value()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == torch::kInt64 && trace->numel() >= 6 * 64,
                "mla_decode: trace must be an int64 CUDA tensor of 384 entries");
    l.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  if (last_slot.has_value()) {
    CHECK_I32(*last_slot); CHECK_ON(q, *last_slot); CHECK_CONTIG(*last_slot);
    TORCH_CHECK(last_slot->numel() >= B, "mla_decode: last_slot shorter than the batch");
    l.last_slot = last_slot->data_ptr<int>();
  }
  l.scale = (float)scale;
  l.err = err_word();
  l.stream = stream();
  if (ks) {
    TORCH_CHECK(!trace.has_value(), "mla_decode: no trace for the fp8 cache kernel");
    l.kv_scales = ks;
    sp::mla_decode_fp8(l);
  } else {
    sp::mla_decode(l);
  }
}

void kv8_gather(const Tensor& cache8, const Tensor& scales, const Tensor& idx, const Tensor& out) {
  CHECK_CUDA(cache8); CHECK_I32(idx); CHECK_BF16(out); CHECK_CONTIG(idx); CHECK_CONTIG(out);
  CHECK_ON(cache8, idx); CHECK_ON(cache8, out);
  const float* ks = kv8_scales(cache8, scales, "kv8_gather");
  TORCH_CHECK(ks, "kv8_gather: the cache must be fp8");
  TORCH_CHECK(out.dim() == 2 && out.size(1) == 576 && out.size(0) >= idx.numel(), "kv8_gather: out [n, 576]");
  const c10::cuda::CUDAGuard guard(cache8.device());
  sp::kv8_gather(cache8.data_ptr(), ks, idx.data_ptr<int>(), out.data_ptr(), (int)idx.numel(), stream());
}

// Stream-K MLA decode (mla_decode_sk.cu); scratch sizes from mla_sk_segments / mla_sk_heads_per_cta.
void mla_decode_sk(const Tensor& q, const Tensor& cache, const Tensor& block_table, const Tensor& context_lens,
                   const Tensor& out, const Tensor& o_part, const Tensor& lse_part, const Tensor& counters,
                   double scale, bool early, const c10::optional<Tensor>& trace) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_BF16(cache); CHECK_I32(block_table); CHECK_I32(context_lens); CHECK_BF16(out);
  CHECK_CONTIG(q); CHECK_CONTIG(block_table); CHECK_CONTIG(out); CHECK_CONTIG(context_lens);
  CHECK_F32(o_part); CHECK_F32(lse_part); CHECK_I32(counters);
  CHECK_ON(q, cache); CHECK_ON(q, block_table); CHECK_ON(q, context_lens); CHECK_ON(q, out);
  CHECK_ON(q, o_part); CHECK_ON(q, lse_part); CHECK_ON(q, counters);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 576, "q: [B, H, 576]");
  TORCH_CHECK(cache.size(-1) == 576 && cache.stride(-1) == 1 && cache.is_contiguous(), "cache rows of 576");
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(sp::mla_sk_supported((int)B, (int)H), "mla_decode_sk: unsupported batch / head count");
  TORCH_CHECK(block_table.size(0) >= B && context_lens.numel() >= B, "mla_decode_sk: block table / lengths too short");
  TORCH_CHECK(out.numel() >= B * H * 512, "mla_decode_sk: output too small");
  const c10::cuda::CUDAGuard guard(q.device());
  const int sms = num_sms();
  const int64_t hg = sp::mla_sk_heads_per_cta((int)H);
  const int64_t segs = sp::mla_sk_segments((int)B, (int)H, sms);
  TORCH_CHECK(o_part.numel() >= segs * hg * 512 && lse_part.numel() >= segs * hg, "mla_decode_sk: scratch too small");
  TORCH_CHECK(counters.numel() >= (H / hg) * B, "mla_decode_sk: counters too small");
  sp::MlaDecodeLaunch l;
  l.q = q.data_ptr();
  l.cache = cache.data_ptr();
  l.num_slots = cache.numel() / 576;
  l.block_table = block_table.data_ptr<int>();
  l.max_blocks = (int)block_table.size(1);
  l.context_lens = context_lens.data_ptr<int>();
  l.out = out.data_ptr();
  l.o_part = o_part.data_ptr<float>();
  l.lse_part = lse_part.data_ptr<float>();
  l.counters = counters.data_ptr<int>();
  l.B = (int)B;
  l.H = (int)H;
  l.scale = (float)scale;
  l.early = early ? 1 : 0;
  if (trace.has_value()) {
    CHECK_ON(q, *trace);
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->numel() >= 4 * 64,
                "mla_decode_sk: trace must be an int64 CUDA tensor of 256 entries");
    l.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  l.err = err_word();
  l.stream = stream();
  sp::mla_decode_sk(l, sms);
}

void prefill_attention(const Tensor& q, const Tensor& k, const Tensor& kpe, const Tensor& v, const Tensor& o,
                       const Tensor& cu_q, const Tensor& cu_k, int64_t max_q, double scale, bool causal,
                       int64_t impl) {
  // q [Tq, H, 192], k [Tk, H, >=128] (nope part at offset 0), kpe [Tk, 64], v [Tk, H, 128], o [Tq, H, 128]
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_BF16(k); CHECK_BF16(kpe); CHECK_BF16(v); CHECK_BF16(o);
  CHECK_I32(cu_q); CHECK_I32(cu_k);
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3 && o.dim() == 3 && kpe.dim() == 2, "prefill shapes");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1 && o.stride(2) == 1 && kpe.stride(1) == 1,
              "prefill: unit innermost stride");
  const c10::cuda::CUDAGuard guard(q.device());
  sp::PrefillAttnLaunch l;
  l.q = q.data_ptr(); l.q_tok = q.stride(0); l.q_head = q.stride(1);
  l.k = k.data_ptr(); l.k_tok = k.stride(0); l.k_head = k.stride(1);
  l.kpe = kpe.data_ptr(); l.kpe_tok = kpe.stride(0);
  l.v = v.data_ptr(); l.v_tok = v.stride(0); l.v_head = v.stride(1);
  l.o = o.data_ptr(); l.o_tok = o.stride(0); l.o_head = o.stride(1);
  l.cu_q = cu_q.data_ptr<int>(); l.cu_k = cu_k.data_ptr<int>();
  l.B = (int)cu_q.size(0) - 1;
  l.H = (int)q.size(1);
  l.max_q = (int)max_q;
  l.scale = (float)scale;
  l.causal = causal ? 1 : 0;
  l.q_rows = q.size(0);
  l.k_rows = k.size(0);
  TORCH_CHECK(kpe.size(0) == k.size(0) && v.size(0) == k.size(0), "prefill: k / kpe / v rows differ");
  TORCH_CHECK(cu_q.numel() == cu_k.numel(), "prefill: cu_q / cu_k lengths differ");
  l.impl = (int)impl;
  l.err = err_word();
  l.stream = stream();
  sp::prefill_attention(l);
}

void moe_topk(const Tensor& logits, const c10::optional<Tensor>& bias, const Tensor& ids, const Tensor& w,
              int64_t n_shared, int64_t scoring, bool renorm, double scaling, int64_t T, int64_t E,
              int64_t slab_stride, int64_t splits, int64_t n_group, int64_t topk_group, bool group_top2) {
  // logits: [T, E] fp32, or the split-K workspace holding `splits` [T, E] slabs slab_stride apart
  CHECK_CUDA(logits); CHECK_F32(logits); CHECK_CONTIG(logits); CHECK_I32(ids); CHECK_F32(w);
  const c10::cuda::CUDAGuard guard(logits.device());
  const float* b = nullptr;
  if (bias.has_value()) { CHECK_F32(*bias); b = bias->data_ptr<float>(); }
  sp::moe_topk(logits.data_ptr<float>(), slab_stride, (int)splits, b, ids.data_ptr<int>(), w.data_ptr<float>(), (int)T,
               (int)E, (int)(ids.size(1) - n_shared), (int)n_shared, (int)scoring, renorm ? 1 : 0, (float)scaling,
               (int)n_group, (int)topk_group, group_top2 ? 1 : 0, stream());
}

// Router top-k with the logits computed in the kernel: x [T, H] bf16, gate [E, H] bf16.
void moe_route(const Tensor& x, const Tensor& gate, const c10::optional<Tensor>& bias, const Tensor& ids,
               const Tensor& w, int64_t n_shared, int64_t scoring, bool renorm, double scaling, int64_t n_group,
               int64_t topk_group, bool group_top2) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(gate); CHECK_CONTIG(gate); CHECK_I32(ids); CHECK_F32(w);
  TORCH_CHECK(x.stride(1) == 1 && x.size(1) == gate.size(1), "moe_route: x [T, H] and gate [E, H]");
  TORCH_CHECK(ids.size(0) >= x.size(0) && w.size(0) >= x.size(0), "moe_route: outputs too small");
  const c10::cuda::CUDAGuard guard(x.device());
  const float* b = nullptr;
  if (bias.has_value()) { CHECK_F32(*bias); b = bias->data_ptr<float>(); }
  sp::moe_topk(nullptr, 0, 1, b, ids.data_ptr<int>(), w.data_ptr<float>(), (int)x.size(0), (int)gate.size(0),
               (int)(ids.size(1) - n_shared), (int)n_shared, (int)scoring, renorm ? 1 : 0, (float)scaling,
               (int)n_group, (int)topk_group, group_top2 ? 1 : 0, stream(), x.data_ptr(), x.stride(0),
               gate.data_ptr(), (int)x.size(1));
}

void slab_add_rmsnorm(const Tensor& slabs, int64_t stride, int64_t splits, const Tensor& residual, const Tensor& w,
                      const Tensor& out, double eps) {
  CHECK_CUDA(slabs); CHECK_F32(slabs); CHECK_BF16(residual); CHECK_CONTIG(residual); CHECK_BF16(w); CHECK_BF16(out);
  const c10::cuda::CUDAGuard guard(slabs.device());
  sp::slab_add_rmsnorm(slabs.data_ptr<float>(), stride, (int)splits, residual.data_ptr(), w.data_ptr(),
                       out.data_ptr(), out.stride(0), (int)residual.size(0), (int)residual.size(1), (float)eps,
                       stream());
}

void mla_decode_prep(const c10::optional<Tensor>& slabs, int64_t stride, int64_t splits,
                     const c10::optional<Tensor>& src, const Tensor& norm_w, const Tensor& positions,
                     const Tensor& cos_sin, const Tensor& slot_mapping, const Tensor& cache,
                     const c10::optional<Tensor>& q_nope_out, const Tensor& q_lat, int64_t T, int64_t dn,
                     int64_t q_off, int64_t kv_off, int64_t row_len, double eps,
                     const c10::optional<Tensor>& kv_scales) {
  CHECK_I32(positions); CHECK_F32(cos_sin); CHECK_I32(slot_mapping);
  float* ks = kv8_scales(cache, kv_scales, "mla_decode_prep");
  CHECK_BF16(q_lat); CHECK_CONTIG(q_lat);
  void* qn = nullptr;
  if (q_nope_out.has_value()) {
    CHECK_BF16(*q_nope_out); CHECK_CONTIG(*q_nope_out);
    qn = q_nope_out->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(q_lat.device());
  const float* sl = nullptr;
  const void* sr = nullptr;
  long long lds = 0;
  if (slabs.has_value()) { CHECK_F32(*slabs); sl = slabs->data_ptr<float>(); }
  if (src.has_value()) { CHECK_BF16(*src); TORCH_CHECK(src->stride(1) == 1, "src rows"); sr = src->data_ptr(); lds = src->stride(0); }
  TORCH_CHECK((sl != nullptr) != (sr != nullptr), "mla_decode_prep: exactly one of slabs / src");
  const int H = (int)q_lat.size(1), W = (int)q_lat.size(2);
  const int kvl = (int)norm_w.size(0);
  sp::mla_decode_prep(sl, stride, (int)splits, sr, lds, norm_w.data_ptr(), positions.data_ptr<int>(),
                      cos_sin.data_ptr<float>(), slot_mapping.data_ptr<int>(), cache.data_ptr(), ks, qn,
                      q_lat.data_ptr(), (int)T, H, (int)dn, W - kvl, kvl, (int)q_off, (int)kv_off, (int)row_len,
                      (float)eps, stream());
}

void combine_add_rmsnorm(const Tensor& y, const Tensor& inv_pos, const Tensor& w, const Tensor& residual,
                         const Tensor& gamma, const Tensor& out, int64_t k, double eps,
                         const c10::optional<Tensor>& shared) {
  CHECK_CUDA(y); CHECK_BF16(y); CHECK_I32(inv_pos); CHECK_F32(w); CHECK_BF16(residual); CHECK_CONTIG(residual);
  CHECK_BF16(gamma); CHECK_BF16(out);
  const int64_t T = residual.size(0);
  const void* sh = nullptr;
  long long ldsh = 0;
  int nsh = 0;
  if (shared.has_value()) {  // [S * T, H] rows s * T + t: the shared experts' outputs, weight 1
    CHECK_BF16(*shared); CHECK_ON(y, *shared);
    TORCH_CHECK(shared->dim() == 2 && shared->stride(1) == 1 && shared->size(1) == residual.size(1) && T > 0 &&
                    shared->size(0) % T == 0,
                "combine_add_rmsnorm: shared rows [S * T, H]");
    sh = shared->data_ptr();
    ldsh = shared->stride(0);
    nsh = (int)(shared->size(0) / T);
  }
  const c10::cuda::CUDAGuard guard(y.device());
  sp::combine_add_rmsnorm(y.data_ptr(), y.stride(0), inv_pos.data_ptr<int>(), w.data_ptr<float>(), residual.data_ptr(),
                          gamma.data_ptr(), out.data_ptr(), out.stride(0), (int)T, (int)k,
                          (int)residual.size(1), (float)eps, stream(), sh, ldsh, nsh);
}

Tensor split_workspace() {
  float* w = split_ws();
  auto opts = torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA, c10::cuda::current_device());
  return torch::from_blob(w, {kSplitWsFloats}, opts);
}

int64_t moe_align(const Tensor& topk_ids, int64_t num_experts, int64_t block_n, const Tensor& grp_rows,
               const Tensor& grp_tiles, const Tensor& sorted_tok, const Tensor& inv_pos, const Tensor& work) {
  CHECK_CUDA(topk_ids); CHECK_I32(topk_ids); CHECK_CONTIG(topk_ids);
  CHECK_I32(grp_rows); CHECK_I32(grp_tiles); CHECK_I32(sorted_tok); CHECK_I32(inv_pos); CHECK_I32(work);
  TORCH_CHECK(work.numel() >= 129 * num_experts, "moe_align: work holds 129 x experts ints");
  const c10::cuda::CUDAGuard guard(topk_ids.device());
  return sp::moe_align(topk_ids.data_ptr<int>(), (int)topk_ids.size(0), (int)topk_ids.size(1), (int)num_experts,
                (int)block_n, grp_rows.data_ptr<int>(), grp_tiles.data_ptr<int>(), sorted_tok.data_ptr<int>(),
                inv_pos.data_ptr<int>(), work.data_ptr<int>(), stream());
}

void gather_rows(const Tensor& x, const Tensor& idx, const Tensor& out) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(out); CHECK_I32(idx);
  const c10::cuda::CUDAGuard guard(x.device());
  sp::gather_rows(x.data_ptr(), x.stride(0), idx.data_ptr<int>(), out.data_ptr(), out.stride(0), (int)idx.size(0),
                  (int)x.size(1), stream());
}

void silu_mul(const Tensor& h, const Tensor& out) {
  CHECK_CUDA(h); CHECK_BF16(h); CHECK_BF16(out);
  TORCH_CHECK(h.size(1) == 2 * out.size(1), "silu_mul: h is [R, 2F], out [R, F]");
  const c10::cuda::CUDAGuard guard(h.device());
  sp::silu_mul(h.data_ptr(), h.stride(0), out.data_ptr(), out.stride(0), (int)out.size(0), (int)out.size(1),
               stream());
}

void moe_combine(const Tensor& y, const Tensor& inv_pos, const Tensor& w, const c10::optional<Tensor>& add,
                 const Tensor& out, int64_t k) {
  CHECK_CUDA(y); CHECK_BF16(y); CHECK_I32(inv_pos); CHECK_F32(w); CHECK_BF16(out);
  const c10::cuda::CUDAGuard guard(y.device());
  const void* a = nullptr;
  long long lda = 0;
  if (add.has_value()) { CHECK_BF16(*add); a = add->data_ptr(); lda = add->stride(0); }
  sp::moe_combine(y.data_ptr(), y.stride(0), inv_pos.data_ptr<int>(), w.data_ptr<float>(), a, lda, out.data_ptr(),
                  out.stride(0), (int)out.size(0), (int)k, (int)out.size(1), stream());
}

void embedding(const Tensor& table, const Tensor& ids, const Tensor& out) {
  CHECK_CUDA(table); CHECK_BF16(table); CHECK_I32(ids); CHECK_BF16(out);
  const c10::cuda::CUDAGuard guard(table.device());
  sp::embedding(table.data_ptr(), table.stride(0), ids.data_ptr<int>(), out.data_ptr(), out.stride(0),
                (int)ids.size(0), (int)table.size(1), stream());
}

void sample_tokens(const Tensor& logits, double temperature, int64_t seed, int64_t offset, const Tensor& out_ids,
                   const c10::optional<Tensor>& out_logit, const c10::optional<Tensor>& row_temp,
                   const c10::optional<Tensor>& row_key) {
  CHECK_CUDA(logits); CHECK_BF16(logits); CHECK_I32(out_ids);
  TORCH_CHECK(logits.stride(1) == 1, "logits rows must be contiguous");
  const c10::cuda::CUDAGuard guard(logits.device());
  float* ol = nullptr;
  if (out_logit.has_value()) { CHECK_F32(*out_logit); ol = out_logit->data_ptr<float>(); }
  const float* rt = nullptr;
  const unsigned long long* rk = nullptr;
  TORCH_CHECK(row_temp.has_value() == row_key.has_value(), "sample_tokens: row_temp and row_key go together");
  if (row_temp.has_value()) {
    CHECK_F32(*row_temp); CHECK_CONTIG(*row_temp); CHECK_CONTIG(*row_key);
    TORCH_CHECK(row_key->scalar_type() == torch::kInt64, "row_key must be int64");
    TORCH_CHECK(row_temp->numel() >= logits.size(0) && row_key->numel() >= logits.size(0),
                "sample_tokens: fewer row parameters than logits rows");
    rt = row_temp->data_ptr<float>();
    rk = reinterpret_cast<const unsigned long long*>(row_key->data_ptr<int64_t>());
  }
  sp::sample_tokens(logits.data_ptr(), logits.stride(0), (int)logits.size(0), (int)logits.size(1),
                    (float)temperature, (unsigned long long)seed, (unsigned long long)offset, out_ids.data_ptr<int>(),
                    ol, rt, rk, stream());
}

void gather_prev_tokens(const Tensor& ids, const Tensor& prev, int64_t n) {
  CHECK_CUDA(ids); CHECK_I32(ids); CHECK_I32(prev); CHECK_CONTIG(ids); CHECK_CONTIG(prev);
  TORCH_CHECK(n >= 0 && n <= ids.numel(), "gather_prev_tokens: n out of range");
  const c10::cuda::CUDAGuard guard(ids.device());
  sp::gather_prev_tokens(ids.data_ptr<int>(), prev.data_ptr<int>(), (int)n, (int)prev.numel(), stream());
}

void dequant_nvfp4(const Tensor& packed, const Tensor& scales, double tensor_scale, const Tensor& out) {
  CHECK_CUDA(packed); CHECK_ON(packed, scales); CHECK_ON(packed, out);
  CHECK_CONTIG(packed); CHECK_CONTIG(scales); CHECK_CONTIG(out);
  TORCH_CHECK(packed.scalar_type() == at::kByte && scales.scalar_type() == at::kByte, "dequant_nvfp4: uint8 inputs");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16, "dequant_nvfp4: bf16 output");
  TORCH_CHECK(out.numel() == packed.numel() * 2 && out.numel() == scales.numel() * 16, "dequant_nvfp4: sizes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(packed.data_ptr()) % 8 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "dequant_nvfp4: alignment");
  const c10::cuda::CUDAGuard guard(packed.device());
  sp::dequant_nvfp4(packed.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(), (float)tensor_scale, out.numel(),
                    out.data_ptr(), stream());
}

void spec_verify(const Tensor& draft, const Tensor& target, double p_accept, int64_t seed, int64_t offset,
                 const Tensor& accepted, const Tensor& committed) {
  CHECK_CUDA(draft); CHECK_I32(draft); CHECK_I32(target); CHECK_I32(accepted); CHECK_I32(committed);
  CHECK_ON(draft, target); CHECK_ON(draft, accepted); CHECK_ON(draft, committed);
  CHECK_CONTIG(draft); CHECK_CONTIG(target); CHECK_CONTIG(committed);
  const c10::cuda::CUDAGuard guard(draft.device());
  sp::spec_verify(draft.data_ptr<int>(), target.data_ptr<int>(), (int)draft.size(0), (int)draft.size(1),
                  (float)p_accept, (unsigned long long)seed, (unsigned long long)offset, accepted.data_ptr<int>(),
                  committed.data_ptr<int>(), stream());
}

void spec_finish(const Tensor& tok_rows, const Tensor& tgt_rows, int64_t L, double p_accept, int64_t seed,
                 const Tensor& pos_rows, const Tensor& ctx_rows, const Tensor& slot_rows, const Tensor& block_table,
                 int64_t block_size, const Tensor& accepted, const Tensor& committed,
                 const c10::optional<Tensor>& total_committed) {
  CHECK_CUDA(tok_rows); CHECK_I32(tok_rows); CHECK_I32(tgt_rows); CHECK_I32(pos_rows); CHECK_I32(ctx_rows);
  CHECK_I32(slot_rows); CHECK_I32(block_table); CHECK_I32(accepted); CHECK_I32(committed);
  CHECK_CONTIG(block_table); CHECK_CONTIG(committed);
  const int64_t B = accepted.numel();
  TORCH_CHECK(tok_rows.numel() == (L + 1) * B && tgt_rows.numel() >= (L + 1) * B && pos_rows.numel() == (L + 1) * B &&
                  ctx_rows.numel() == (L + 1) * B && slot_rows.numel() == (L + 1) * B &&
                  committed.numel() == (L + 1) * B && block_table.size(0) >= B,
              "spec_finish: row arrays must hold (L + 1) x B entries");
  unsigned long long* tc = nullptr;
  if (total_committed.has_value()) {
    TORCH_CHECK(total_committed->scalar_type() == at::kLong, "total_committed must be int64");
    tc = reinterpret_cast<unsigned long long*>(total_committed->data_ptr<int64_t>());
  }
  const c10::cuda::CUDAGuard guard(tok_rows.device());
  sp::spec_finish(tok_rows.data_ptr<int>(), tgt_rows.data_ptr<int>(), (int)B, (int)L, (float)p_accept,
                  (unsigned long long)seed, pos_rows.data_ptr<int>(), ctx_rows.data_ptr<int>(),
                  slot_rows.data_ptr<int>(), block_table.data_ptr<int>(), (int)block_table.size(1), (int)block_size,
                  accepted.data_ptr<int>(), committed.data_ptr<int>(), tc, stream());
}

// Verify round of the serving engine: chain acceptance with per-lane budgets.
void spec_chain_commit(const Tensor& tok, const Tensor& tgt, const Tensor& ctx, const Tensor& pos,
                       const Tensor& budget, const Tensor& keys, int64_t L, double p_accept, int64_t seed,
                       const Tensor& committed, const Tensor& counts) {
  CHECK_CUDA(tok); CHECK_I32(tok); CHECK_I32(tgt); CHECK_I32(ctx); CHECK_I32(pos); CHECK_I32(budget);
  CHECK_I32(committed); CHECK_I32(counts);
  TORCH_CHECK(keys.scalar_type() == at::kLong, "keys must be int64");
  for (const Tensor* t : {&tgt, &ctx, &pos, &budget, &keys, &committed, &counts}) { CHECK_ON(tok, *t); CHECK_CONTIG(*t); }
  CHECK_CONTIG(tok);
  const int64_t B = counts.numel();
  TORCH_CHECK(L >= 1 && tok.numel() >= (L + 1) * B && tgt.numel() >= (L + 1) * B && ctx.numel() >= B &&
                  pos.numel() >= B && budget.numel() >= B && keys.numel() >= B && committed.numel() >= (L + 1) * B,
              "spec_chain_commit: row arrays must hold (L + 1) x B entries");
  const c10::cuda::CUDAGuard guard(tok.device());
  sp::spec_chain_commit(tok.data_ptr<int>(), tgt.data_ptr<int>(), ctx.data_ptr<int>(), pos.data_ptr<int>(),
                        budget.data_ptr<int>(), reinterpret_cast<const unsigned long long*>(keys.data_ptr<int64_t>()),
                        (int)B, (int)L, (float)p_accept, (unsigned long long)seed, committed.data_ptr<int>(),
                        counts.data_ptr<int>(), stream());
}

// Verify round of the serving engine: the MTP tree (6 rows per lane) and the KV move
// of an accepted alternate leaf in `cache` [layers, slots, row].
void mtp_tree_commit(const Tensor& tok, const Tensor& tgt, const Tensor& ctx, const Tensor& slots,
                     const Tensor& cache, const Tensor& committed, const Tensor& counts, const Tensor& paths,
                     const c10::optional<Tensor>& aux) {
  CHECK_CUDA(tok); CHECK_I32(tok); CHECK_I32(tgt); CHECK_I32(ctx); CHECK_I32(slots);
  TORCH_CHECK(cache.element_size() == 2 || cache.element_size() == 1, "mtp_tree_commit: bf16 or fp8 cache");
  CHECK_I32(committed); CHECK_I32(counts); CHECK_I32(paths); CHECK_CONTIG(cache);
  for (const Tensor* t : {&tgt, &ctx, &slots, &cache, &committed, &counts, &paths}) CHECK_ON(tok, *t);
  for (const Tensor* t : {&tok, &tgt, &ctx, &slots, &committed, &counts, &paths}) CHECK_CONTIG(*t);
  TORCH_CHECK(cache.dim() == 3, "cache: [layers, slots, row]");
  const int64_t B = counts.numel();
  TORCH_CHECK(tok.numel() >= 6 * B && tgt.numel() >= 6 * B && slots.numel() >= 6 * B && ctx.numel() >= B &&
                  committed.numel() >= 6 * B && paths.numel() >= B,
              "mtp_tree_commit: row arrays must hold 6 x B entries");
  const c10::cuda::CUDAGuard guard(tok.device());
  // rows move as 2-byte units (an fp8 row of 576 bytes is 288 of them)
  const int es = (int)cache.element_size();
  TORCH_CHECK((cache.size(2) * es) % 2 == 0 && (cache.stride(0) * es) % 2 == 0, "mtp_tree_commit: row bytes");
  float* ax = nullptr;
  long long ax_stride = 0;
  int ax_row = 0;
  if (aux.has_value()) {
    CHECK_F32(*aux); CHECK_CONTIG(*aux); CHECK_ON(tok, *aux);
    TORCH_CHECK(aux->dim() == 3 && aux->size(0) == cache.size(0) && aux->size(1) == cache.size(1),
                "mtp_tree_commit: aux [layers, slots, k]");
    ax = aux->data_ptr<float>();
    ax_stride = aux->stride(0);
    ax_row = (int)aux->size(2);
  }
  sp::mtp_tree_commit(tok.data_ptr<int>(), tgt.data_ptr<int>(), ctx.data_ptr<int>(), slots.data_ptr<int>(), (int)B,
                      cache.data_ptr(), cache.stride(0) * es / 2, (int)cache.size(0), (int)(cache.size(2) * es / 2),
                      committed.data_ptr<int>(), counts.data_ptr<int>(), paths.data_ptr<int>(), stream(), ax,
                      ax_stride, ax_row);
}

void top2_rows(const Tensor& logits, const Tensor& out0, const Tensor& out1) {
  CHECK_CUDA(logits); CHECK_BF16(logits); CHECK_I32(out0); CHECK_I32(out1);
  CHECK_ON(logits, out0); CHECK_ON(logits, out1); CHECK_CONTIG(out0); CHECK_CONTIG(out1);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits: [T, V] with unit column stride");
  const int64_t T = logits.size(0);
  TORCH_CHECK(out0.numel() >= T && out1.numel() >= T, "top2_rows: outputs shorter than the rows");
  const c10::cuda::CUDAGuard guard(logits.device());
  sp::top2_rows(logits.data_ptr(), logits.stride(0), (int)T, (int)logits.size(1), out0.data_ptr<int>(),
                out1.data_ptr<int>(), stream());
}

void kv_blocks_copy(const Tensor& cache, const Tensor& blocks, const Tensor& staging, int64_t block_size,
                    bool to_staging) {
  // cache [layers, slots, row] bf16 (contiguous); staging [n, layers, block_size, row] bf16
  CHECK_CUDA(cache); CHECK_BF16(cache); CHECK_CONTIG(cache); CHECK_BF16(staging); CHECK_CONTIG(staging);
  CHECK_I32(blocks); CHECK_CONTIG(blocks);
  TORCH_CHECK(cache.dim() == 3 && cache.size(1) % block_size == 0, "kv_blocks_copy: cache [layers, slots, row]");
  const int64_t n = blocks.numel(), L = cache.size(0), row = cache.size(2);
  TORCH_CHECK(staging.numel() >= n * L * block_size * row, "kv_blocks_copy: staging too small");
  const c10::cuda::CUDAGuard guard(cache.device());
  sp::kv_blocks_copy(cache.data_ptr(), cache.stride(0), blocks.data_ptr<int>(), (int)n, staging.data_ptr(), (int)L,
                     (int)block_size, (int)row, to_staging ? 1 : 0, stream());
}

void phase_mark(const Tensor& stamps, const c10::optional<Tensor>& totals, int64_t slot, int64_t prev) {
  TORCH_CHECK(stamps.is_cuda() && stamps.scalar_type() == at::kLong && slot >= 0 && slot < stamps.numel(),
              "phase_mark: stamps must be a CUDA int64 tensor holding the slot");
  unsigned long long* tot = nullptr;
  if (totals.has_value()) {
    TORCH_CHECK(totals->scalar_type() == at::kLong && totals->numel() == stamps.numel(), "phase_mark: totals");
    tot = reinterpret_cast<unsigned long long*>(totals->data_ptr<int64_t>());
  }
  const c10::cuda::CUDAGuard guard(stamps.device());
  TORCH_CHECK(prev < stamps.numel(), "phase_mark: previous slot");
  sp::phase_mark(reinterpret_cast<unsigned long long*>(stamps.data_ptr<int64_t>()), tot, (int)slot, (int)prev,
                 stream());
}

void decode_advance(const Tensor& out_ids, const Tensor& ids, const Tensor& pos, const Tensor& ctx,
                    const Tensor& slots, const Tensor& block_table, int64_t block_size) {
  CHECK_CUDA(ids); CHECK_I32(out_ids); CHECK_I32(ids); CHECK_I32(pos); CHECK_I32(ctx); CHECK_I32(slots);
  CHECK_I32(block_table); CHECK_CONTIG(block_table);
  const c10::cuda::CUDAGuard guard(ids.device());
  sp::decode_advance(out_ids.data_ptr<int>(), ids.data_ptr<int>(), pos.data_ptr<int>(), ctx.data_ptr<int>(),
                     slots.data_ptr<int>(), block_table.data_ptr<int>(), (int)block_table.size(1), (int)ids.size(0),
                     (int)block_size, stream());
}

// ---------------------------------------------------------------- DSA selection
void paged_slots(const Tensor& block_table, const Tensor& lens, const c10::optional<Tensor>& positions,
                 int64_t rows, int64_t block_size, const Tensor& slots) {
  CHECK_CUDA(block_table); CHECK_I32(block_table); CHECK_I32(lens); CHECK_I32(slots); CHECK_CONTIG(block_table);
  const int64_t B = block_table.size(0);
  TORCH_CHECK(lens.numel() >= B && slots.numel() >= B * rows, "paged_slots: lengths / output too small");
  const int* pp = nullptr;
  if (positions.has_value()) {
    CHECK_I32(*positions); CHECK_CONTIG(*positions);
    TORCH_CHECK(positions->numel() >= B * rows, "paged_slots: positions too small");
    pp = positions->data_ptr<int>();
  }
  const c10::cuda::CUDAGuard guard(block_table.device());
  sp::paged_slots(block_table.data_ptr<int>(), (int)block_table.size(1), lens.data_ptr<int>(), pp, (int)B, (int)rows,
                  (int)block_size, slots.data_ptr<int>(), stream());
}

void dsa_topk(const Tensor& raw, const Tensor& w, const Tensor& lens, int64_t topk, const Tensor& scores,
              const Tensor& out, const Tensor& counts) {
  CHECK_CUDA(raw); CHECK_F32(raw); CHECK_F32(w); CHECK_I32(lens); CHECK_F32(scores); CHECK_I32(out);
  CHECK_I32(counts); CHECK_CONTIG(raw); CHECK_CONTIG(w); CHECK_CONTIG(scores); CHECK_CONTIG(out);
  TORCH_CHECK(raw.dim() == 3, "dsa_topk: raw [B, heads, rows]");
  const int64_t B = raw.size(0), Hi = raw.size(1), rows = raw.size(2);
  TORCH_CHECK(w.numel() >= B * Hi && lens.numel() >= B && scores.numel() >= B * rows && out.numel() >= B * topk &&
                  counts.numel() >= B,
              "dsa_topk: operand too small");
  const c10::cuda::CUDAGuard guard(raw.device());
  sp::dsa_topk(raw.data_ptr<float>(), w.data_ptr<float>(), (int)B, (int)Hi, (int)rows, lens.data_ptr<int>(),
               (int)topk, scores.data_ptr<float>(), out.data_ptr<int>(), counts.data_ptr<int>(), stream());
}

// ---------------------------------------------------------------- raw device memory
// Untyped device allocations for native components that keep their own ledger
// (stage modules): pointers cross as integers.
int64_t raw_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, (size_t)bytes) == cudaSuccess, "raw_alloc: cudaMalloc failed");
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}
void raw_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>((uintptr_t)ptr)); }
int64_t raw_zero(int64_t ptr, int64_t bytes) {
  return cudaMemset(reinterpret_cast<void*>((uintptr_t)ptr), 0, (size_t)bytes) == cudaSuccess ? 0 : 17;
}
int64_t raw_copy(int64_t dst, int64_t src, int64_t bytes) {
  return cudaMemcpy(reinterpret_cast<void*>((uintptr_t)dst), reinterpret_cast<const void*>((uintptr_t)src),
                    (size_t)bytes, cudaMemcpyDefault) == cudaSuccess
             ? 0
             : 17;
}

// ---------------------------------------------------------------- expert parallel
// One cudaMalloc per rank holds every EP region; its IPC handle is exchanged
// over the process group and each peer maps it (cudaIpcOpenMemHandle), so the
// kernels address all ranks' buffers directly.
Tensor ep_alloc(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, nbytes) == cudaSuccess, "ep: buffer allocation failed");
  TORCH_CHECK(cudaMemset(p, 0, nbytes) == cudaSuccess, "ep: buffer clear failed");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

py::bytes ep_ipc_handle(const Tensor& buf) {
  CHECK_CUDA(buf);
  const c10::cuda::CUDAGuard guard(buf.device());
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, buf.data_ptr()) == cudaSuccess, "ep: cudaIpcGetMemHandle failed");
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ep_ipc_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "ep: bad IPC handle size");
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "ep: cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void ep_ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

sp::EpArgs ep_args(const std::vector<int64_t>& v) {
  TORCH_CHECK((int)v.size() == sp::EP_ARGS_WORDS, "ep: argument vector must hold ", sp::EP_ARGS_WORDS, " words");
  sp::EpArgs a{};
  int i = 0;
  for (int r = 0; r < sp::EP_MAX_RANKS; ++r) a.base[r] = (unsigned long long)v[i++];
  a.off_ctrl = v[i++]; a.off_nch = v[i++]; a.off_meta = v[i++]; a.off_rows = v[i++]; a.off_comb = v[i++];
  a.world = (int)v[i++]; a.rank = (int)v[i++]; a.cap = (int)v[i++]; a.H = (int)v[i++]; a.kk = (int)v[i++];
  a.n_routed = (int)v[i++]; a.experts_per_rank = (int)v[i++]; a.n_shared = (int)v[i++]; a.moe_layers = (int)v[i++];
  a.max_chunks = (int)v[i++];
  a.fp8 = (int)v[i++]; a.row_words = v[i++]; a.shared_local = (int)v[i++];
  for (int r = 0; r < a.world; ++r) TORCH_CHECK(a.base[r] != 0 && a.base[r] % 256 == 0, "ep: bad rank base pointer");
  return a;
}

void ep_dispatch(const Tensor& x, const Tensor& ids, const std::vector<int64_t>& args, const Tensor& epoch,
                 int64_t layer) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_I32(ids); CHECK_CONTIG(ids);
  TORCH_CHECK(x.stride(1) == 1 && x.stride(0) % 8 == 0, "ep: x rows must be contiguous and 16-byte aligned");
  TORCH_CHECK(epoch.scalar_type() == at::kLong, "ep: epoch must be int64");
  const c10::cuda::CUDAGuard guard(x.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(x.size(1) == a.H && ids.numel() == x.size(0) * a.kk, "ep: shape mismatch");
  sp::ep_dispatch(x.data_ptr(), x.stride(0), ids.data_ptr<int>(), (int)x.size(0), a, epoch.data_ptr<int64_t>(),
                  (int)layer, stream());
}

void ep_recv_align(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, int64_t bn,
                   const Tensor& grp_rows, const Tensor& grp_tiles, const Tensor& src_row, const Tensor& comb_dst,
                   int64_t budget_cycles) {
  CHECK_I32(grp_rows); CHECK_I32(grp_tiles); CHECK_I32(src_row); CHECK_I32(comb_dst);
  const c10::cuda::CUDAGuard guard(grp_rows.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(grp_rows.numel() >= a.experts_per_rank + a.n_shared + 1, "ep: grp_rows too small");
  TORCH_CHECK(src_row.numel() >= (int64_t)a.world * a.cap * std::min(a.kk, a.experts_per_rank + a.n_shared),
              "ep: pair buffers too small");
  sp::ep_recv_align(a, epoch.data_ptr<int64_t>(), (int)layer, (int)bn, grp_rows.data_ptr<int>(),
                    grp_tiles.data_ptr<int>(), src_row.data_ptr<int>(), comb_dst.data_ptr<int>(), budget_cycles,
                    err_word(), stream());
}

void ep_gather(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, const Tensor& total,
               const Tensor& src_row, const Tensor& xs, int64_t budget_cycles) {
  CHECK_BF16(xs); CHECK_CONTIG(xs); CHECK_I32(src_row); CHECK_I32(total);
  const c10::cuda::CUDAGuard guard(xs.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(xs.size(1) == a.H, "ep: xs width");
  sp::ep_gather(a, epoch.data_ptr<int64_t>(), (int)layer, total.data_ptr<int>(), src_row.data_ptr<int>(),
                xs.data_ptr(), budget_cycles, err_word(), num_sms(), stream());
}

void ep_gather_fp8(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, const Tensor& total,
                   const Tensor& src_row, const Tensor& xq, const Tensor& xs_scale, int64_t budget_cycles) {
  CHECK_FP8(xq); CHECK_F32(xs_scale); CHECK_I32(src_row); CHECK_I32(total);
  TORCH_CHECK(xq.dim() == 2 && xq.stride(1) == 1 && xs_scale.dim() == 2 && xs_scale.stride(1) == 1, "ep: 2-D views");
  const c10::cuda::CUDAGuard guard(xq.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(xq.size(1) == a.H && xs_scale.size(0) * 128 == a.H, "ep: fp8 gather shapes");
  TORCH_CHECK(xq.size(0) >= src_row.numel() && xs_scale.stride(0) >= xq.size(0), "ep: fp8 gather capacity");
  sp::ep_gather_fp8(a, epoch.data_ptr<int64_t>(), (int)layer, total.data_ptr<int>(), src_row.data_ptr<int>(),
                    xq.data_ptr(), xq.stride(0), xs_scale.data_ptr<float>(), xs_scale.stride(0), budget_cycles,
                    err_word(), num_sms(), stream());
}

void ep_combine_send(const Tensor& y, const Tensor& total, const Tensor& comb_dst, const std::vector<int64_t>& args,
                     const Tensor& epoch, int64_t layer) {
  CHECK_BF16(y); CHECK_CONTIG(y); CHECK_I32(total); CHECK_I32(comb_dst);
  const c10::cuda::CUDAGuard guard(y.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(y.size(1) == a.H, "ep: y width");
  sp::ep_combine_send(y.data_ptr(), total.data_ptr<int>(), comb_dst.data_ptr<int>(), a, epoch.data_ptr<int64_t>(),
                      (int)layer, stream());
}

void ep_combine_add_rmsnorm(const std::vector<int64_t>& args, const Tensor& epoch, int64_t layer, const Tensor& w,
                            const Tensor& residual, const Tensor& gamma, const Tensor& out, double eps,
                            int64_t budget_cycles, const c10::optional<Tensor>& y_shared) {
  CHECK_F32(w); CHECK_CONTIG(w); CHECK_BF16(residual); CHECK_CONTIG(residual); CHECK_BF16(gamma); CHECK_BF16(out);
  TORCH_CHECK(out.stride(1) == 1 && out.stride(0) % 8 == 0, "ep: out rows must be contiguous and 16-byte aligned");
  const c10::cuda::CUDAGuard guard(residual.device());
  const sp::EpArgs a = ep_args(args);
  TORCH_CHECK(residual.size(1) == a.H && w.numel() == residual.size(0) * a.kk, "ep: combine shape mismatch");
  const void* ys = nullptr;
  if (y_shared.has_value()) {
    CHECK_BF16(*y_shared); CHECK_CONTIG(*y_shared);
    TORCH_CHECK(y_shared->numel() >= (int64_t)a.n_shared * residual.size(0) * a.H, "ep: shared rows too small");
    ys = y_shared->data_ptr();
  }
  sp::ep_combine_add_rmsnorm(a, epoch.data_ptr<int64_t>(), (int)layer, w.data_ptr<float>(), residual.data_ptr(),
                             gamma.data_ptr(), out.data_ptr(), out.stride(0), (int)residual.size(0), (float)eps,
                             budget_cycles, err_word(), ys, stream());
}

void ep_advance(const Tensor& epoch) {
  TORCH_CHECK(epoch.scalar_type() == at::kLong && epoch.is_cuda(), "ep: epoch must be a CUDA int64 tensor");
  const c10::cuda::CUDAGuard guard(epoch.device());
  sp::ep_advance(epoch.data_ptr<int64_t>(), stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of the sparkpipe_rs_b200 serving engine";
  m.def("gemm", &gemm);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("mla_kv_write", &mla_kv_write);
  m.def("rope_q", &rope_q);
  m.def("quant_fp8_block", &quant_fp8_block);
  m.def("gemm_fp8", &gemm_fp8);
  m.def("quant_act_fp8", &quant_act_fp8);
  m.def("quant_weight_fp8", &quant_weight_fp8);
  m.def("mla_decode", &mla_decode);
  m.def("kv8_gather", &kv8_gather);
  m.def("mla_fp8_ctas_per_sm", [](int64_t heads) { return sp::mla_fp8_ctas_per_sm((int)heads); });
  m.def("mla_decode_sk", &mla_decode_sk);
  m.def("mla_sk_supported", [](int64_t B, int64_t H) { return sp::mla_sk_supported((int)B, (int)H); });
  m.def("mla_sk_heads_per_cta", [](int64_t H) { return sp::mla_sk_heads_per_cta((int)H); });
  m.def("mla_sk_segments", [](int64_t B, int64_t H, int64_t sms) { return sp::mla_sk_segments((int)B, (int)H, (int)sms); });
  m.def("prefill_attention", &prefill_attention);
  m.def("moe_topk", &moe_topk);
  m.def("moe_align", &moe_align);
  m.def("gather_rows", &gather_rows);
  m.def("silu_mul", &silu_mul);
  m.def("moe_combine", &moe_combine);
  m.def("embedding", &embedding);
  m.def("sample_tokens", &sample_tokens);
  m.def("gather_prev_tokens", &gather_prev_tokens);
  m.def("dequant_nvfp4", &dequant_nvfp4);
  m.def("spec_verify", &spec_verify);
  m.def("decode_advance", &decode_advance);
  m.def("spec_finish", &spec_finish);
  m.def("grouped_gemm_tm", &grouped_gemm_tm);
  m.def("spec_chain_commit", &spec_chain_commit);
  m.def("mtp_tree_commit", &mtp_tree_commit);
  m.def("top2_rows", &top2_rows);
  m.def("phase_mark", &phase_mark);
  m.def("kv_blocks_copy", &kv_blocks_copy);
  m.def("slab_add_rmsnorm", &slab_add_rmsnorm);
  m.def("mla_decode_prep", &mla_decode_prep);
  m.def("combine_add_rmsnorm", &combine_add_rmsnorm);
  m.def("split_workspace", &split_workspace);
  m.def("status_word", &status_word);
  m.def("clear_status", &clear_status);
  m.def("num_sms", &num_sms);
  m.def("mla_ctas_per_sm", [](int64_t heads, int64_t impl) { return sp::mla_ctas_per_sm((int)heads, (int)impl); },
        py::arg("heads"), py::arg("impl") = 0);
  m.def("mla_stage_tokens", []() { return sp::mla_stage_tokens(); });
  m.def("kernel_attributes", []() {
    std::vector<sp::KernelAttr> v;
    sp::kernel_attrs_gemm(v);
    sp::kernel_attrs_fp8(v);
    sp::kernel_attrs_mla(v);
    sp::kernel_attrs_mla8(v);
    sp::kernel_attrs_mla_sk(v);
    sp::kernel_attrs_prefill(v);
    sp::kernel_attrs_moe(v);
    py::list out;
    for (const auto& a : v) {
      py::dict d;
      d["name"] = a.name;
      d["registers"] = a.regs;
      d["local_bytes"] = a.local_bytes;
      d["static_smem"] = a.static_smem;
      d["max_threads"] = a.max_threads;
      d["ptx_version"] = a.ptx_version;
      d["binary_version"] = a.binary_version;
      out.append(d);
    }
    return out;
  });
  m.def("moe_route", &moe_route);
  m.def("paged_slots", &paged_slots);
  m.def("dsa_topk", &dsa_topk);
  m.def("raw_alloc", &raw_alloc);
  m.def("raw_free", &raw_free);
  m.def("raw_zero", &raw_zero);
  m.def("raw_copy", &raw_copy);
  m.def("ep_alloc", &ep_alloc);
  m.def("ep_ipc_handle", &ep_ipc_handle);
  m.def("ep_ipc_open", &ep_ipc_open);
  m.def("ep_ipc_close", &ep_ipc_close);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_recv_align", &ep_recv_align);
  m.def("ep_gather", &ep_gather);
  m.def("ep_gather_fp8", &ep_gather_fp8);
  m.def("ep_combine_send", &ep_combine_send);
  m.def("ep_combine_add_rmsnorm", &ep_combine_add_rmsnorm);
  m.def("ep_advance", &ep_advance);
  m.def("gemm_tp", &gemm_tp);
  m.def("tp_rs_add_rmsnorm", &tp_rs_add_rmsnorm);
  m.def("tp_ag_send", &tp_ag_send);
  m.attr("TP_ARGS_WORDS") = kTpArgsWords;
  m.attr("EP_ARGS_WORDS") = sp::EP_ARGS_WORDS;
  m.attr("EP_MAX_RANKS") = sp::EP_MAX_RANKS;
  m.attr("EP_CHUNK_TOKENS") = sp::EP_CHUNK_TOKENS;
  m.attr("EP_COMBINE_CTAS") = sp::EP_COMBINE_CTAS;
}
