// Expert-parallel MoE dispatch / combine over NVLink peer memory, sm_100a.
//
// Layout: attention is data-parallel (each rank owns its tokens), routed
// experts are split evenly over the W ranks (rank r owns experts
// [r*El, (r+1)*El)), shared experts are replicated and run locally. Every rank
// maps every peer's EP buffer (CUDA IPC), so the kernels below move data with
// plain loads / stores to peer addresses; there are no copy engines, no NCCL
// calls and no host synchronisation in the per-layer path.
//
// Transport: every word that crosses to a peer is a 64-bit store of
// (payload:32 | tag:32) with tag = low 32 bits of (epoch + 1). A reader polls
// the word itself until the tag matches, so a 64-bit single-copy-atomic store
// is both the data and its own arrival flag: no system-scope fences, no flag
// words, no ordering between words. (A system-scope fence costs microseconds
// on this machine; a layer needs several of them otherwise.) Rows therefore
// travel at twice their size, which is irrelevant at decode batch sizes.
//
// Per MoE layer (epoch e = step * layers_per_step + layer, buffer parity e & 1):
//   ep_dispatch            grid (destination, 8-token chunk): stores each token
//                          routed to that destination once (row + (token, local
//                          expert, k-slot) list) into the chunk's own slots of
//                          this source's region there, plus the chunk's row
//                          count (and, for chunk 0, the chunk count).
//   ep_recv_align          one CTA: reads every source's counts and lists and
//                          builds the expert-sorted pair list, the grouped-GEMM
//                          tile schedule and the combine destinations.
//   ep_gather              received rows -> expert-sorted bf16 rows (local HBM).
//   grouped GEMMs          (gemm_tcgen05.cu) gate/up with fused SwiGLU, then down.
//   ep_combine_send        grid (destination, 16): each output row goes straight
//                          into its source rank's combine slot (token, k-slot).
//   ep_combine_add_rmsnorm the source sums its k slots per token (router
//                          weights), adds the residual and applies the next
//                          RMSNorm, reading the slots as they arrive.
//
// Why two buffers suffice: rank A dispatches layer e+2 only after it consumed
// the combine of layer e+1, which rank B sent only after it received layer e+1
// (and so layer e) completely. Every poll is bounded (clock64 budget); on a
// timeout the kernel records kErrWaitTimeoutPeer in the status word, empties
// its outputs and returns, so the context stays usable and the host raises.
//
// Reference: the fused-MoE and expert-queue seams of the reference
// (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:321-342,
// V/model-families/glm52 expert queue); the reference has no multi-GPU expert
// all-to-all of its own.
#include "common.cuh"
#include "launch.h"
#include "ll.cuh"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {
SP_DEVI uint8_t* rank_base(const EpArgs& a, int r) { return reinterpret_cast<uint8_t*>(a.base[r]); }
// (rows in chunk c of source src) on rank r
SP_DEVI u64* ctrl_word(const EpArgs& a, int r, int buf, int src, int c) {
  return reinterpret_cast<u64*>(rank_base(a, r) + a.off_ctrl) + (int64_t(buf) * EP_MAX_RANKS + src) * a.max_chunks + c;
}
// (chunks the source sent this epoch) on rank r
SP_DEVI u64* nch_word(const EpArgs& a, int r, int buf, int src) {
  return reinterpret_cast<u64*>(rank_base(a, r) + a.off_nch) + buf * EP_MAX_RANKS + src;
}
SP_DEVI u64* meta_words(const EpArgs& a, int r, int buf, int src, int row) {
  return reinterpret_cast<u64*>(rank_base(a, r) + a.off_meta) +
         ((int64_t(buf) * a.world + src) * a.cap + row) * (2 + 2 * a.kk);
}
SP_DEVI u64* row_words(const EpArgs& a, int r, int buf, int src, int row) {
  return reinterpret_cast<u64*>(rank_base(a, r) + a.off_rows) + ((int64_t(buf) * a.world + src) * a.cap + row) * a.row_words;
}
SP_DEVI u64* comb_words(const EpArgs& a, int r, int buf, int slot) {
  return reinterpret_cast<u64*>(rank_base(a, r) + a.off_comb) + (int64_t(buf) * a.cap * a.kk + slot) * (a.H / 2);
}

SP_DEVI uint32_t epoch_tag(const int64_t* epoch_ptr, const EpArgs& a, int layer, int* buf) {
  const u64 e = u64(*epoch_ptr) * a.moe_layers + layer;
  *buf = int(e & 1);
  return uint32_t(e + 1);
}

// One warp sends one bf16 row as tagged words: lane handles 8 columns (16 B in,
// 4 words = 32 B out) per step; all of a lane's loads are issued before its
// stores so the row costs one load latency, not one per step.
constexpr int EP_ROW_STEPS = 8;  // 16-byte steps per lane held in registers per pass (2048 columns)
SP_DEVI void warp_send_row(u64* dst, const bf16* src, int H, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  const int n = H / 8;
  for (int c0 = 0; c0 < n; c0 += 32 * EP_ROW_STEPS) {
    uint4 v[EP_ROW_STEPS];
#pragma unroll
    for (int u = 0; u < EP_ROW_STEPS; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < n) v[u] = __ldcg(s + c);
    }
#pragma unroll
    for (int u = 0; u < EP_ROW_STEPS; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < n) {
        st_ll2(dst + 4 * c, ll_word(v[u].x, tag), ll_word(v[u].y, tag));
        st_ll2(dst + 4 * c + 2, ll_word(v[u].z, tag), ll_word(v[u].w, tag));
      }
    }
  }
}

// fp8 transport: one warp quantises and sends one row. Block b of 128 columns
// becomes 32 payload words (4 e4m3 per lane) at words [32b, 32b + 32) and one
// scale word at H/4 + b; the quantiser is the one quant_act_fp8 uses.
SP_DEVI void warp_send_row_fp8(u64* dst, const bf16* src, int H, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  const int nb = H / 128;
  for (int b0 = 0; b0 < nb; b0 += EP_ROW_STEPS) {
    uint2 v[EP_ROW_STEPS];
#pragma unroll
    for (int u = 0; u < EP_ROW_STEPS; ++u)
      if (b0 + u < nb) v[u] = __ldcg(reinterpret_cast<const uint2*>(src + (b0 + u) * 128 + lane * 4));
#pragma unroll
    for (int u = 0; u < EP_ROW_STEPS; ++u) {
      const int b = b0 + u;
      if (b >= nb) break;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
      const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
      float scale;
      const uint32_t q = warp_quant_e4m3_block(f0.x, f0.y, f1.x, f1.y, scale);
      st_ll(dst + b * 32 + lane, ll_word(q, tag));
      if (lane == 0) st_ll(dst + H / 4 + b, ll_word(__float_as_uint(scale), tag));
    }
  }
}
}  // namespace

// grid (W destinations, C chunks of EP_CHUNK_TOKENS tokens), 256 threads
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                          const int* __restrict__ ids, int T, EpArgs a,
                                                          const int64_t* __restrict__ epoch_ptr, int layer) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int d = blockIdx.x, c = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_tok[EP_CHUNK_TOKENS], s_n;
  if (warp == 0) {
    const int t = c * EP_CHUNK_TOKENS + lane;
    int n = 0;
    int le[EP_MAX_KK], jj[EP_MAX_KK];
    if (lane < EP_CHUNK_TOKENS && t < T) {
      for (int j = 0; j < a.kk; ++j) {
        const int id = ids[t * a.kk + j];
        if (a.shared_local && id >= a.n_routed) continue;  // computed on this rank, not dispatched
        const int dd = id >= a.n_routed ? a.rank : id / a.experts_per_rank;
        if (dd == d) {
          le[n] = id >= a.n_routed ? a.experts_per_rank + (id - a.n_routed) : id - dd * a.experts_per_rank;
          jj[n] = j;
          ++n;
        }
      }
    }
    const unsigned mask = __ballot_sync(0xffffffffu, n > 0);
    if (n > 0) {
      const int pos = __popc(mask & ((1u << lane) - 1));
      u64* m = meta_words(a, d, buf, a.rank, c * EP_CHUNK_TOKENS + pos);
      st_ll(m, ll_word(uint32_t(t), tag));
      st_ll(m + 1, ll_word(uint32_t(n), tag));
      for (int q = 0; q < n; ++q) {
        st_ll(m + 2 + q, ll_word(uint32_t(le[q]), tag));
        st_ll(m + 2 + a.kk + q, ll_word(uint32_t(jj[q]), tag));
      }
      s_tok[pos] = t;
    }
    if (lane == 0) {
      s_n = __popc(mask);
      st_ll(ctrl_word(a, d, buf, a.rank, c), ll_word(uint32_t(__popc(mask)), tag));
      if (c == 0) st_ll(nch_word(a, d, buf, a.rank), ll_word(gridDim.y, tag));
    }
  }
  __syncthreads();
  const int n = s_n;
  for (int i = warp; i < n; i += blockDim.x / 32) {
    u64* dst = row_words(a, d, buf, a.rank, c * EP_CHUNK_TOKENS + i);
    if (a.fp8) warp_send_row_fp8(dst, x + int64_t(s_tok[i]) * ldx, a.H, tag);
    else warp_send_row(dst, x + int64_t(s_tok[i]) * ldx, a.H, tag);
  }
}

constexpr int EP_ALIGN_MAX_E = 1024;

SP_DEVI void ep_scan(const int* counts, int E, int bn, int* grp_rows, int* grp_tiles, int* cursor) {
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
    const int u = __shfl_up_sync(0xffffffffu, ri, o);
    const int v = __shfl_up_sync(0xffffffffu, ti, o);
    if (lane >= o) { ri += u; ti += v; }
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

__global__ void __launch_bounds__(1024) ep_recv_align_kernel(EpArgs a, const int64_t* __restrict__ epoch_ptr,
                                                             int layer, int bn, int* __restrict__ grp_rows,
                                                             int* __restrict__ grp_tiles, int* __restrict__ src_row,
                                                             int* __restrict__ comb_dst, long long budget,
                                                             int* __restrict__ gerr) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int El = a.experts_per_rank + a.n_shared;
  __shared__ int cnt[EP_ALIGN_MAX_E], cur[EP_ALIGN_MAX_E], nch[EP_MAX_RANKS], s_rows;
  extern __shared__ int s_count[];  // [world][max_chunks] rows per (source, chunk)
  bool ok = true;
  if (threadIdx.x < a.world) {
    const int v = int(poll_ll(nch_word(a, a.rank, buf, threadIdx.x), tag, budget, ok, gerr));
    nch[threadIdx.x] = v < 1 ? 1 : (v > a.max_chunks ? a.max_chunks : v);
  }
  if (__syncthreads_and(ok)) {
    for (int i = threadIdx.x; i < a.world * a.max_chunks && ok; i += blockDim.x) {
      const int s = i / a.max_chunks, c = i % a.max_chunks;
      s_count[i] = c < nch[s] ? int(poll_ll(ctrl_word(a, a.rank, buf, s, c), tag, budget, ok, gerr)) : 0;
    }
    for (int i = threadIdx.x; i < El; i += blockDim.x) cnt[i] = 0;
    if (threadIdx.x == 0) {
      int m = 0;
      for (int s = 0; s < a.world; ++s) m = nch[s] > m ? nch[s] : m;
      s_rows = m * EP_CHUNK_TOKENS;  // row slots to scan per source
    }
  }
  ok = __syncthreads_and(ok);
  const int rows = ok ? s_rows : 0, total = a.world * rows;
  // pass 1: histogram of local experts over every received (row, entry), all sources at once
  for (int i = threadIdx.x; i < total && ok; i += blockDim.x) {
    const int s = i / rows, r = i % rows;
    if (r % EP_CHUNK_TOKENS >= s_count[s * a.max_chunks + r / EP_CHUNK_TOKENS]) continue;
    const u64* m = meta_words(a, a.rank, buf, s, r);
    // one batch of loads for the row's whole list, then the (rare) late words
    u64 w[2 + EP_MAX_KK];
#pragma unroll
    for (int q = 0; q < 2 + EP_MAX_KK; ++q)
      if (q < 2 + a.kk) w[q] = ld_ll(m + q);
    const int n = tag_of(w[1]) == tag ? int(uint32_t(w[1])) : int(poll_ll(m + 1, tag, budget, ok, gerr));
#pragma unroll
    for (int q = 0; q < EP_MAX_KK; ++q) {
      if (q >= n || !ok) break;
      const int le = tag_of(w[2 + q]) == tag ? int(uint32_t(w[2 + q])) : int(poll_ll(m + 2 + q, tag, budget, ok, gerr));
      if (ok && le < El) atomicAdd(&cnt[le], 1);
    }
  }
  if (!__syncthreads_and(ok)) {
    for (int i = threadIdx.x; i <= El; i += blockDim.x) grp_rows[i] = grp_tiles[i] = 0;
    if (threadIdx.x == 0) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
    return;
  }
  if (threadIdx.x < 32) ep_scan(cnt, El, bn, grp_rows, grp_tiles, cur);
  __syncthreads();
  // pass 2: every word has arrived (pass 1 saw them); scatter to expert-sorted positions
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int s = i / rows, r = i % rows;
    if (r % EP_CHUNK_TOKENS >= s_count[s * a.max_chunks + r / EP_CHUNK_TOKENS]) continue;
    const u64* m = meta_words(a, a.rank, buf, s, r);
    bool ok2 = true;
    const int tok = int(poll_ll(m, tag, budget, ok2, gerr)), n = int(uint32_t(ld_ll(m + 1)));
    for (int q = 0; q < n; ++q) {
      const int le = int(uint32_t(ld_ll(m + 2 + q)));
      if (le >= El) continue;
      const int p = atomicAdd(&cur[le], 1);
      src_row[p] = s * a.cap + r;
      comb_dst[p] = (s << 20) | (tok * a.kk + int(poll_ll(m + 2 + a.kk + q, tag, budget, ok2, gerr)));
    }
    if (!ok2) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
  }
}

// received rows (tagged words) -> expert-sorted bf16 rows; one warp per row
__global__ void __launch_bounds__(256) ep_gather_kernel(EpArgs a, const int64_t* __restrict__ epoch_ptr, int layer,
                                                        const int* __restrict__ total, const int* __restrict__ src_row,
                                                        bf16* __restrict__ xs, long long budget,
                                                        int* __restrict__ gerr) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int n = *total;
  const u64* base = row_words(a, a.rank, buf, 0, 0);
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  bool ok = true;
  const int nc = a.H / 8;
  for (int p = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); p < n && ok; p += warps) {
    const u64* src = base + int64_t(src_row[p]) * a.row_words;
    uint4* dst = reinterpret_cast<uint4*>(xs + int64_t(p) * a.H);
    for (int c0 = 0; c0 < nc && ok; c0 += 32 * EP_ROW_STEPS) {
      u64 w[EP_ROW_STEPS][4];
      // issue every load of this pass first, then check tags (re-poll only the late ones)
#pragma unroll
      for (int u = 0; u < EP_ROW_STEPS; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < nc) {
          ld_ll2(src + 4 * c, w[u][0], w[u][1]);
          ld_ll2(src + 4 * c + 2, w[u][2], w[u][3]);
        }
      }
#pragma unroll
      for (int u = 0; u < EP_ROW_STEPS; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= nc) continue;
        uint32_t v[4];
        if (tag_of(w[u][0]) == tag && tag_of(w[u][1]) == tag && tag_of(w[u][2]) == tag && tag_of(w[u][3]) == tag) {
          v[0] = uint32_t(w[u][0]); v[1] = uint32_t(w[u][1]); v[2] = uint32_t(w[u][2]); v[3] = uint32_t(w[u][3]);
        } else if (!poll_ll4(src + 4 * c, tag, budget, v, gerr)) {
          ok = false;
          break;
        }
        dst[c] = make_uint4(v[0], v[1], v[2], v[3]);
      }
    }
  }
  if (!ok) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
}

// fp8 transport: received rows -> expert-sorted e4m3 rows + K-block-major scales;
// one warp per row, lanes move 2 payload words (8 e4m3) per step.
__global__ void __launch_bounds__(256) ep_gather_fp8_kernel(EpArgs a, const int64_t* __restrict__ epoch_ptr, int layer,
                                                            const int* __restrict__ total,
                                                            const int* __restrict__ src_row, uint8_t* __restrict__ xq,
                                                            long long ldq, float* __restrict__ xs_scale, long long lds,
                                                            long long budget, int* __restrict__ gerr) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int n = *total;
  const u64* base = row_words(a, a.rank, buf, 0, 0);
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  const int npairs = a.H / 8;  // word pairs of payload
  const int nb = a.H / 128;
  bool ok = true;
  for (int p = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); p < n && ok; p += warps) {
    const u64* src = base + int64_t(src_row[p]) * a.row_words;
    uint2* dst = reinterpret_cast<uint2*>(xq + int64_t(p) * ldq);
    for (int c0 = 0; c0 < npairs && ok; c0 += 32 * EP_ROW_STEPS) {
      u64 w[EP_ROW_STEPS][2];
#pragma unroll
      for (int u = 0; u < EP_ROW_STEPS; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < npairs) ld_ll2(src + 2 * c, w[u][0], w[u][1]);
      }
#pragma unroll
      for (int u = 0; u < EP_ROW_STEPS; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= npairs) continue;
        uint32_t v0, v1;
        if (tag_of(w[u][0]) == tag && tag_of(w[u][1]) == tag) {
          v0 = uint32_t(w[u][0]);
          v1 = uint32_t(w[u][1]);
        } else {
          bool ok2 = true;
          v0 = poll_ll(src + 2 * c, tag, budget, ok2, gerr);
          v1 = poll_ll(src + 2 * c + 1, tag, budget, ok2, gerr);
          if (!ok2) { ok = false; break; }
        }
        dst[c] = make_uint2(v0, v1);
      }
    }
    for (int b = lane; b < nb && ok; b += 32) {
      bool ok2 = true;
      const uint32_t sc = poll_ll(src + a.H / 4 + b, tag, budget, ok2, gerr);
      if (!ok2) { ok = false; break; }
      xs_scale[int64_t(b) * lds + p] = __uint_as_float(sc);
    }
  }
  if (!ok) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
}

// grid (W destinations, EP_COMBINE_CTAS): output rows whose source is rank d go
// straight into d's combine slots as tagged words
__global__ void __launch_bounds__(256) ep_combine_send_kernel(const bf16* __restrict__ y, const int* __restrict__ total,
                                                              const int* __restrict__ comb_dst, EpArgs a,
                                                              const int64_t* __restrict__ epoch_ptr, int layer) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int d = blockIdx.x, c = blockIdx.y;
  const int n = *total;
  const int wpc = blockDim.x / 32;
  for (int p = c * wpc + (threadIdx.x >> 5); p < n; p += EP_COMBINE_CTAS * wpc) {
    const int dst = comb_dst[p];
    if ((dst >> 20) == d) warp_send_row(comb_words(a, d, buf, dst & 0xFFFFF), y + int64_t(p) * a.H, a.H, tag);
  }
}

// res[t] += sum_j w[t, j] * slot(t, j); out[t] = rmsnorm(res[t]) * gamma, with the
// slots read as they arrive. Same per-element arithmetic and reduction order as
// combine_add_rmsnorm (moe.cu), so results are bit-identical to the local path.
__global__ void __launch_bounds__(256) ep_combine_add_rmsnorm_kernel(
    EpArgs a, const int64_t* __restrict__ epoch_ptr, int layer, const float* __restrict__ w, bf16* __restrict__ res,
    const bf16* __restrict__ gamma, bf16* __restrict__ out, long long ldo, float eps, long long budget,
    int* __restrict__ gerr, const bf16* __restrict__ y_shared, int T) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = epoch_tag(epoch_ptr, a, layer, &buf);
  const int t = blockIdx.x, k = a.kk, H = a.H;
  __shared__ float s_w[EP_MAX_KK];
  __shared__ float part[8];
  if (threadIdx.x < k) s_w[threadIdx.x] = w[t * k + threadIdx.x];
  __syncthreads();
  bf16* rr = res + (long long)t * H;
  float v[4][8];
  float ss = 0.f;
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // issue the loads of every slot first, then consume them in slot order
      // slots of shared experts computed here (shared_local) come from y_shared
      const int k_remote = a.shared_local ? k - a.n_shared : k;
      u64 w[EP_MAX_KK][4];
#pragma unroll
      for (int j = 0; j < EP_MAX_KK; ++j)
        if (j < k_remote) {
          const u64* p = comb_words(a, a.rank, buf, t * k + j) + c / 2;
          ld_ll2(p, w[j][0], w[j][1]);
          ld_ll2(p + 2, w[j][2], w[j][3]);
        }
#pragma unroll
      for (int j = 0; j < EP_MAX_KK; ++j) {
        if (j >= k) break;
        uint32_t raw[4];
        if (j >= k_remote) {
          const uint4 u = *reinterpret_cast<const uint4*>(y_shared + ((long long)(j - k_remote) * T + t) * H + c);
          raw[0] = u.x; raw[1] = u.y; raw[2] = u.z; raw[3] = u.w;
        } else if (tag_of(w[j][0]) == tag && tag_of(w[j][1]) == tag && tag_of(w[j][2]) == tag && tag_of(w[j][3]) == tag) {
          raw[0] = uint32_t(w[j][0]); raw[1] = uint32_t(w[j][1]); raw[2] = uint32_t(w[j][2]); raw[3] = uint32_t(w[j][3]);
        } else if (!ok || !poll_ll4(comb_words(a, a.rank, buf, t * k + j) + c / 2, tag, budget, raw, gerr)) {
          ok = false;
          raw[0] = raw[1] = raw[2] = raw[3] = 0u;
        }
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(raw);
        float yv[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          yv[2 * q] = f.x;
          yv[2 * q + 1] = f.y;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += s_w[j] * yv[e];
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
  if (!ok) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float inv = rsqrtf(tot / H + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float g[8], o[8];
      ld_bf16x8(gamma + c, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * inv * g[e];
      st_bf16x8(out + (long long)t * ldo + c, o);
    }
  }
}

__global__ void ep_advance_kernel(int64_t* epoch_ptr) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0 && blockIdx.x == 0) *epoch_ptr += 1;
}

// ------------------------------------------------------------------ host entry points
static void check_args(const EpArgs& a) {
  if (a.world < 1 || a.world > EP_MAX_RANKS) throw std::runtime_error("ep: world size must be 1..8");
  if (a.kk < 1 || a.kk > EP_MAX_KK) throw std::runtime_error("ep: top-k + shared must be 1..16");
  if (a.H % 8 || a.H > 8192) throw std::runtime_error("ep: hidden size must be a multiple of 8, at most 8192");
  if (a.experts_per_rank + a.n_shared > EP_ALIGN_MAX_E) throw std::runtime_error("ep: too many local experts");
  if (a.cap >= (1 << 20) / a.kk) throw std::runtime_error("ep: token capacity too large for the slot encoding");
  if (a.cap % EP_CHUNK_TOKENS || a.max_chunks != a.cap / EP_CHUNK_TOKENS)
    throw std::runtime_error("ep: capacity must be whole token chunks");
  const long long need = a.fp8 ? a.H / 4 + ((a.H / 128 + 1) & ~1) : a.H / 2;
  if (a.fp8 && a.H % 128) throw std::runtime_error("ep: the fp8 transport needs H % 128 == 0");
  if (a.row_words != need) throw std::runtime_error("ep: row stride does not match the transport");
}

void ep_dispatch(const void* x, int64_t ldx, const int* ids, int T, const EpArgs& a, const int64_t* epoch, int layer,
                 cudaStream_t s) {
  check_args(a);
  if (T > a.cap) throw std::runtime_error("ep: more tokens than the buffer capacity");
  const int chunks = T > 0 ? (T + EP_CHUNK_TOKENS - 1) / EP_CHUNK_TOKENS : 1;
  launch_k(ep_dispatch_kernel, dim3(a.world, chunks), dim3(256), 0, s, static_cast<const bf16*>(x), ldx, ids, T, a,
           epoch, layer);
}

void ep_recv_align(const EpArgs& a, const int64_t* epoch, int layer, int bn, int* grp_rows, int* grp_tiles,
                   int* src_row, int* comb_dst, long long budget, int* err, cudaStream_t s) {
  check_args(a);
  const int smem = a.world * a.max_chunks * (int)sizeof(int);
  if (smem > 160 * 1024) throw std::runtime_error("ep: too many token chunks for the receive kernel");
  if (smem > 32 * 1024) set_smem_bytes(ep_recv_align_kernel, 160 * 1024);
  launch_k(ep_recv_align_kernel, dim3(1), dim3(1024), smem, s, a, epoch, layer, bn, grp_rows, grp_tiles, src_row,
           comb_dst, budget, err);
}

void ep_gather(const EpArgs& a, const int64_t* epoch, int layer, const int* total, const int* src_row, void* xs,
               long long budget, int* err, int num_sms, cudaStream_t s) {
  launch_k(ep_gather_kernel, dim3(num_sms), dim3(256), 0, s, a, epoch, layer, total, src_row, static_cast<bf16*>(xs),
           budget, err);
}

void ep_gather_fp8(const EpArgs& a, const int64_t* epoch, int layer, const int* total, const int* src_row, void* xq,
                   long long ldq, float* xs_scale, long long lds, long long budget, int* err, int num_sms,
                   cudaStream_t s) {
  check_args(a);
  if (!a.fp8) throw std::runtime_error("ep: fp8 gather on a bf16 transport");
  launch_k(ep_gather_fp8_kernel, dim3(num_sms), dim3(256), 0, s, a, epoch, layer, total, src_row,
           static_cast<uint8_t*>(xq), ldq, xs_scale, lds, budget, err);
}

void ep_combine_send(const void* y, const int* total, const int* comb_dst, const EpArgs& a, const int64_t* epoch,
                     int layer, cudaStream_t s) {
  launch_k(ep_combine_send_kernel, dim3(a.world, EP_COMBINE_CTAS), dim3(256), 0, s, static_cast<const bf16*>(y), total,
           comb_dst, a, epoch, layer);
}

void ep_combine_add_rmsnorm(const EpArgs& a, const int64_t* epoch, int layer, const float* topk_w, void* residual,
                            const void* gamma, void* out, long long ldo, int T, float eps, long long budget, int* err,
                            const void* y_shared, cudaStream_t s) {
  check_args(a);
  if (T <= 0) return;
  if (T > a.cap) throw std::runtime_error("ep: more tokens than the buffer capacity");
  if (a.shared_local && a.n_shared > 0 && !y_shared)
    throw std::runtime_error("ep: the shared experts' rows are needed when they run locally");
  launch_k(ep_combine_add_rmsnorm_kernel, dim3(T), dim3(256), 0, s, a, epoch, layer, topk_w,
           static_cast<bf16*>(residual), static_cast<const bf16*>(gamma), static_cast<bf16*>(out), ldo, eps, budget,
           err, static_cast<const bf16*>(y_shared), T);
}

void ep_advance(int64_t* epoch, cudaStream_t s) { launch_k(ep_advance_kernel, dim3(1), dim3(32), 0, s, epoch); }

}  // namespace sp
