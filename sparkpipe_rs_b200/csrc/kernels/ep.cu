// Expert-parallel MoE dispatch / combine over NVLink peer memory, sm_100a.
//
// Layout: attention is data-parallel (each rank owns its tokens), routed
// experts are split evenly over the W ranks (rank r owns experts
// [r*El, (r+1)*El)), shared experts are replicated and run locally. Every rank
// maps every peer's EP buffer (CUDA IPC), so the kernels below move data with
// plain 16-byte loads / stores to peer addresses; there are no copy engines,
// no NCCL calls and no host synchronisation in the per-layer path.
//
// Per MoE layer (epoch e = step * moe_layers + layer, buffer parity e & 1):
//   ep_dispatch     one CTA per local token: for each distinct destination rank
//                   of its top-k experts, reserve a row in that rank's receive
//                   region for this source, store the hidden row and its
//                   (token, local expert, k-slot) list there. The last CTA
//                   publishes the per-destination row counts and raises each
//                   destination's flag (release, system scope).
//   ep_recv_align   one CTA: waits (bounded) for all W flags, builds the
//                   expert-sorted pair list of everything received, the
//                   grouped-GEMM tile schedule and the combine destinations.
//   ep_gather       copies received rows into expert-sorted order (local HBM).
//   grouped GEMMs   (gemm_tcgen05.cu) gate/up with fused SwiGLU, then down.
//   ep_combine_send stores each output row straight into its source rank's
//                   combine buffer at (token, k-slot); the last CTA raises the
//                   combine flag on every rank.
//   ep_wait         waits (bounded) for all W combine flags; the weighted sum is
//                   fused into the next residual add + RMSNorm (moe.cu).
//
// Why two buffers suffice: rank A dispatches layer e+2 only after it consumed
// the combine of layer e+1, which rank B sent only after gathering layer e+1
// (and so layer e). Every wait is bounded (clock64 budget); on a timeout the
// kernel records kErrWaitTimeoutPeer in the status word, empties its outputs
// and returns, so the context stays usable and the host raises.
//
// Reference: the fused-MoE and expert-queue seams of the reference
// (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:321-342,
// V/model-families/glm52 expert queue); the reference has no multi-GPU expert
// all-to-all of its own.
#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {
SP_DEVI void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
SP_DEVI uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
SP_DEVI uint8_t* rank_base(const EpArgs& a, int r) { return reinterpret_cast<uint8_t*>(a.base[r]); }
SP_DEVI uint64_t* recv_flag(const EpArgs& a, int r, int buf, int src) {
  return reinterpret_cast<uint64_t*>(rank_base(a, r) + a.off_recv_flag) + buf * EP_MAX_RANKS + src;
}
SP_DEVI uint64_t* comb_flag(const EpArgs& a, int r, int buf, int src) {
  return reinterpret_cast<uint64_t*>(rank_base(a, r) + a.off_comb_flag) + buf * EP_MAX_RANKS + src;
}
SP_DEVI int* recv_count(const EpArgs& a, int r, int buf, int src) {
  return reinterpret_cast<int*>(rank_base(a, r) + a.off_recv_count) + buf * EP_MAX_RANKS + src;
}
SP_DEVI int* recv_meta(const EpArgs& a, int r, int buf, int src, int row) {
  const int mi = 2 + 2 * a.kk;
  return reinterpret_cast<int*>(rank_base(a, r) + a.off_recv_meta) +
         ((int64_t(buf) * a.world + src) * a.cap + row) * mi;
}
SP_DEVI bf16* recv_row(const EpArgs& a, int r, int buf, int src, int row) {
  return reinterpret_cast<bf16*>(rank_base(a, r) + a.off_recv_x) + ((int64_t(buf) * a.world + src) * a.cap + row) * a.H;
}
SP_DEVI bf16* comb_row(const EpArgs& a, int r, int buf, int slot) {
  return reinterpret_cast<bf16*>(rank_base(a, r) + a.off_comb_x) + (int64_t(buf) * a.cap * a.kk + slot) * a.H;
}
SP_DEVI int* local_scratch(const EpArgs& a) { return reinterpret_cast<int*>(rank_base(a, a.rank) + a.off_scratch); }

// 16-byte vector copy of one hidden row (H % 8 == 0), spread over the CTA
SP_DEVI void copy_row(bf16* dst, const bf16* src, int H) {
  const int4* s = reinterpret_cast<const int4*>(src);
  int4* d = reinterpret_cast<int4*>(dst);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = __ldcg(s + c);  // L2: rows written by peers
}

SP_DEVI bool wait_flags(const uint64_t* flags, int n, uint64_t want, long long budget) {
  // thread i < n waits for flag i; returns false on timeout for any
  bool ok = true;
  if (threadIdx.x < n) {
    const long long t0 = clock64();
    while (ld_acquire_sys(flags + threadIdx.x) != want) {
      if (clock64() - t0 > budget) { ok = false; break; }
      __nanosleep(64);
    }
  }
  return __syncthreads_and(ok);
}
}  // namespace

// scratch ints: [0, W) per-destination row cursors, [W] dispatch ticket, [W+1] combine ticket
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                          const int* __restrict__ ids, int T, EpArgs a,
                                                          const int64_t* __restrict__ epoch_ptr, int layer) {
  griddep_wait();
  griddep_launch();
  const uint64_t e = uint64_t(*epoch_ptr) * a.moe_layers + layer;
  const int buf = int(e & 1);
  int* scr = local_scratch(a);
  __shared__ int s_dest[EP_MAX_KK], s_pos[EP_MAX_KK], s_nd;
  const int t = blockIdx.x;
  if (t < T) {
    if (threadIdx.x == 0) {
      int nd = 0;
      int dest_of[EP_MAX_KK], le_of[EP_MAX_KK];
      for (int j = 0; j < a.kk; ++j) {
        const int id = ids[t * a.kk + j];
        int d, le;
        if (id >= a.n_routed) { d = a.rank; le = a.experts_per_rank + (id - a.n_routed); }  // shared: local
        else { d = id / a.experts_per_rank; le = id - d * a.experts_per_rank; }
        dest_of[j] = d;
        le_of[j] = le;
        bool seen = false;
        for (int q = 0; q < nd; ++q) seen |= s_dest[q] == d;
        if (!seen) s_dest[nd++] = d;
      }
      for (int q = 0; q < nd; ++q) {
        const int d = s_dest[q];
        const int pos = atomicAdd(&scr[d], 1);
        s_pos[q] = pos;
        int* m = recv_meta(a, d, buf, a.rank, pos);
        int n = 0;
        for (int j = 0; j < a.kk; ++j)
          if (dest_of[j] == d) { m[2 + n] = le_of[j]; m[2 + a.kk + n] = j; ++n; }
        m[0] = t;
        m[1] = n;
      }
      s_nd = nd;
    }
    __syncthreads();
    for (int q = 0; q < s_nd; ++q) copy_row(recv_row(a, s_dest[q], buf, a.rank, s_pos[q]), x + int64_t(t) * ldx, a.H);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&scr[a.world], 1);
    if (ticket == int(gridDim.x) - 1) {
      __threadfence();
      for (int d = 0; d < a.world; ++d) {
        *recv_count(a, d, buf, a.rank) = atomicExch(&scr[d], 0);
      }
      __threadfence_system();
      for (int d = 0; d < a.world; ++d) st_release_sys(recv_flag(a, d, buf, a.rank), e + 1);
      scr[a.world] = 0;
    }
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
  const uint64_t e = uint64_t(*epoch_ptr) * a.moe_layers + layer;
  const int buf = int(e & 1);
  const int El = a.experts_per_rank + a.n_shared;
  __shared__ int cnt[EP_ALIGN_MAX_E], cur[EP_ALIGN_MAX_E], rows[EP_MAX_RANKS];
  const bool ok = wait_flags(recv_flag(a, a.rank, buf, 0), a.world, e + 1, budget);
  if (!ok) {
    for (int i = threadIdx.x; i <= El; i += blockDim.x) grp_rows[i] = grp_tiles[i] = 0;
    if (threadIdx.x == 0) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
    return;
  }
  for (int i = threadIdx.x; i < El; i += blockDim.x) cnt[i] = 0;
  if (threadIdx.x < a.world) rows[threadIdx.x] = __ldcg(recv_count(a, a.rank, buf, threadIdx.x));
  __syncthreads();
  const int mi = 2 + 2 * a.kk;
  for (int s = 0; s < a.world; ++s) {
    const int* m0 = recv_meta(a, a.rank, buf, s, 0);
    for (int r = threadIdx.x; r < rows[s]; r += blockDim.x) {
      const int* m = m0 + r * mi;
      const int n = __ldcg(m + 1);
      for (int q = 0; q < n; ++q) atomicAdd(&cnt[__ldcg(m + 2 + q)], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) ep_scan(cnt, El, bn, grp_rows, grp_tiles, cur);
  __syncthreads();
  for (int s = 0; s < a.world; ++s) {
    const int* m0 = recv_meta(a, a.rank, buf, s, 0);
    for (int r = threadIdx.x; r < rows[s]; r += blockDim.x) {
      const int* m = m0 + r * mi;
      const int n = __ldcg(m + 1), tok = __ldcg(m);
      for (int q = 0; q < n; ++q) {
        const int p = atomicAdd(&cur[__ldcg(m + 2 + q)], 1);
        src_row[p] = s * a.cap + r;
        comb_dst[p] = (s << 20) | (tok * a.kk + __ldcg(m + 2 + a.kk + q));
      }
    }
  }
}

__global__ void __launch_bounds__(256) ep_gather_kernel(EpArgs a, const int64_t* __restrict__ epoch_ptr, int layer,
                                                        const int* __restrict__ total, const int* __restrict__ src_row,
                                                        bf16* __restrict__ xs) {
  griddep_wait();
  griddep_launch();
  const uint64_t e = uint64_t(*epoch_ptr) * a.moe_layers + layer;
  const int buf = int(e & 1);
  const int n = *total;
  const bf16* base = recv_row(a, a.rank, buf, 0, 0);
  for (int p = blockIdx.x; p < n; p += gridDim.x) copy_row(xs + int64_t(p) * a.H, base + int64_t(src_row[p]) * a.H, a.H);
}

__global__ void __launch_bounds__(256) ep_combine_send_kernel(const bf16* __restrict__ y, const int* __restrict__ total,
                                                              const int* __restrict__ comb_dst, EpArgs a,
                                                              const int64_t* __restrict__ epoch_ptr, int layer) {
  griddep_wait();
  griddep_launch();
  const uint64_t e = uint64_t(*epoch_ptr) * a.moe_layers + layer;
  const int buf = int(e & 1);
  const int n = *total;
  for (int p = blockIdx.x; p < n; p += gridDim.x) {
    const int d = comb_dst[p];
    copy_row(comb_row(a, d >> 20, buf, d & 0xFFFFF), y + int64_t(p) * a.H, a.H);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* scr = local_scratch(a);
    const int ticket = atomicAdd(&scr[a.world + 1], 1);
    if (ticket == int(gridDim.x) - 1) {
      __threadfence_system();
      for (int d = 0; d < a.world; ++d) st_release_sys(comb_flag(a, d, buf, a.rank), e + 1);
      scr[a.world + 1] = 0;
    }
  }
}

__global__ void __launch_bounds__(32) ep_wait_combine_kernel(EpArgs a, const int64_t* __restrict__ epoch_ptr,
                                                             int layer, long long budget, int* __restrict__ gerr) {
  griddep_wait();
  griddep_launch();
  const uint64_t e = uint64_t(*epoch_ptr) * a.moe_layers + layer;
  const int buf = int(e & 1);
  if (!wait_flags(comb_flag(a, a.rank, buf, 0), a.world, e + 1, budget) && threadIdx.x == 0)
    atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
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
  if (a.H % 8) throw std::runtime_error("ep: hidden size must be a multiple of 8");
  if (a.experts_per_rank + a.n_shared > EP_ALIGN_MAX_E) throw std::runtime_error("ep: too many local experts");
  if (a.cap >= (1 << 20) / a.kk) throw std::runtime_error("ep: token capacity too large for the slot encoding");
}

void ep_dispatch(const void* x, int64_t ldx, const int* ids, int T, const EpArgs& a, const int64_t* epoch, int layer,
                 cudaStream_t s) {
  check_args(a);
  if (T > a.cap) throw std::runtime_error("ep: more tokens than the buffer capacity");
  launch_k(ep_dispatch_kernel, dim3(T > 0 ? T : 1), dim3(256), 0, s, static_cast<const bf16*>(x), ldx, ids, T, a,
           epoch, layer);
}

void ep_recv_align(const EpArgs& a, const int64_t* epoch, int layer, int bn, int* grp_rows, int* grp_tiles,
                   int* src_row, int* comb_dst, long long budget, int* err, cudaStream_t s) {
  check_args(a);
  launch_k(ep_recv_align_kernel, dim3(1), dim3(1024), 0, s, a, epoch, layer, bn, grp_rows, grp_tiles, src_row,
           comb_dst, budget, err);
}

void ep_gather(const EpArgs& a, const int64_t* epoch, int layer, const int* total, const int* src_row, void* xs,
               int num_sms, cudaStream_t s) {
  launch_k(ep_gather_kernel, dim3(num_sms * 2), dim3(256), 0, s, a, epoch, layer, total, src_row,
           static_cast<bf16*>(xs));
}

void ep_combine_send(const void* y, const int* total, const int* comb_dst, const EpArgs& a, const int64_t* epoch,
                     int layer, int num_sms, cudaStream_t s) {
  launch_k(ep_combine_send_kernel, dim3(num_sms * 2), dim3(256), 0, s, static_cast<const bf16*>(y), total, comb_dst,
           a, epoch, layer);
}

void ep_wait_combine(const EpArgs& a, const int64_t* epoch, int layer, long long budget, int* err, cudaStream_t s) {
  launch_k(ep_wait_combine_kernel, dim3(1), dim3(32), 0, s, a, epoch, layer, budget, err);
}

void ep_advance(int64_t* epoch, cudaStream_t s) { launch_k(ep_advance_kernel, dim3(1), dim3(32), 0, s, epoch); }

}  // namespace sp
