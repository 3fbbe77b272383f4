// Tensor parallelism over NVLink peer memory, sm_100a: the consumer and producer
// halves of the fused reduce-scatter / all-gather around TP GEMMs.
//
// Layout (sequence parallel): the T tokens of a step are split into W blocks of
// `rows` tokens; rank r owns rows [r*rows, (r+1)*rows) of the residual stream.
//
//   row-parallel GEMM -> RS   the GEMM epilogue (gemm_tcgen05.cu, tp_rs) sends
//                             its fp32 partial of token n as tagged words into
//                             slot (rank, split) of the owner's RS region;
//   tp_rs_add_rmsnorm         the owner sums its W x S slots per element in a fixed
//                             order (deterministic), adds the residual, applies
//                             RMSNorm, and (optionally) all-gathers the normed row:
//                             plain bf16 stores into every rank's AG region at row
//                             rank*rows + t, then system-scope fences and a release
//                             store of the layer's tag into that row's flag;
//   tp_ag_send                the same all-gather of a row block on its own;
//   AG -> column-parallel GEMM the GEMM producer (tp_ag_flags) acquires the flags of
//                             a tile's rows, then TMA-loads B from the AG region.
//
// The reduce-scatter side uses 64-bit tagged stores (ll.cuh) that need neither fences
// nor flags, since its consumer is a plain kernel that polls; the all-gather side is
// read by TMA, which cannot check tags, so it publishes rows with flags instead (one
// fence per thread, all concurrent). Every wait is bounded (status word kErrWaitTimeoutPeer
// on a timeout). Two parity halves per region (epoch e = step * layers_per_step +
// layer, parity e & 1, layers_per_step even) make back-to-back layers race-free.
//
// The reference's TP collective is a recursive-doubling TCP all-reduce of bf16 /
// f32 vectors (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/
// spark_tp_collective.h); these kernels replace it on NVLink with the reduction
// fused into the GEMM epilogue and the next RMSNorm.
#include <cuda_runtime.h>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ll.cuh"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

namespace {

SP_DEVI uint32_t tp_epoch_tag(const int64_t* epoch_ptr, int layers_per_step, int layer, int* buf) {
  const u64 e = u64(*epoch_ptr) * layers_per_step + layer;
  *buf = int(e & 1);
  return uint32_t(e + 1);
}

// Writes 8 bf16 of row `grow` into every rank's AG region (plain 16-byte stores).
SP_DEVI void ag_put8(const TpArgs& a, int buf, int grow, int c, const float* v) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  const uint4 u = *reinterpret_cast<const uint4*>(h);
  const long long off = ((long long)buf * a.world * a.rows + grow) * a.H + c;
  for (int r = 0; r < a.world; ++r) *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.base[r] + a.ag_off) + off) = u;
}

// After every thread of the CTA stored its part of row `grow`: each thread orders its
// own stores at system scope (the fences run concurrently), then the row's flag on
// every rank takes the layer's tag (release).
SP_DEVI void ag_publish(const TpArgs& a, int buf, uint32_t tag, int grow) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long off = (long long)buf * a.world * a.rows + grow;
    for (int r = 0; r < a.world; ++r) {
      u64* f = reinterpret_cast<u64*>(a.base[r] + a.flag_off) + off;
      asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(u64(tag)) : "memory");
    }
  }
}

}  // namespace

// One CTA (256 threads) per owned row t; H <= 8192.
__global__ void __launch_bounds__(256) tp_rs_add_rmsnorm_kernel(TpArgs a, const int64_t* __restrict__ epoch_ptr,
                                                                int layer, int slots, bf16* __restrict__ res,
                                                                const bf16* __restrict__ gamma,
                                                                bf16* __restrict__ out, long long ldo, float eps,
                                                                int ag_layer, long long budget,
                                                                int* __restrict__ gerr) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = tp_epoch_tag(epoch_ptr, a.layers_per_step, layer, &buf);
  const int t = blockIdx.x, H = a.H;
  const u64* rs = reinterpret_cast<const u64*>(a.base[a.rank] + a.rs_off);
  bf16* rr = res + (long long)t * H;
  float v[4][8];
  float ss = 0.f;
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // slots in groups of 4: issue every load of a group, then check the tags (re-poll
      // only late words), then add in slot order
      for (int s0 = 0; s0 < slots; s0 += 4) {
        u64 w[4][8];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (s0 + q < slots) {
            const u64* p = rs + (((long long)buf * slots + s0 + q) * a.rows + t) * H + c;
#pragma unroll
            for (int j = 0; j < 8; j += 2) ld_ll2(p + j, w[q][j], w[q][j + 1]);
          }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (s0 + q >= slots) break;
          const u64* p = rs + (((long long)buf * slots + s0 + q) * a.rows + t) * H + c;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint32_t v = uint32_t(w[q][j]);
            if (tag_of(w[q][j]) != tag) {
              bool ok2 = ok;
              v = ok ? poll_ll(p + j, tag, budget, ok2, gerr) : 0u;
              ok = ok2;
            }
            x[j] += __uint_as_float(v);
          }
        }
      }
      float r[8];
      ld_bf16x8(rr + c, r);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[i][j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(x[j])) + r[j]));
      st_bf16x8(rr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  if (!ok) atomicCAS(gerr, 0, kErrWaitTimeoutPeer);
  __shared__ float part[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float inv = rsqrtf(tot / H + eps);
  int abuf = 0;
  const uint32_t atag = ag_layer >= 0 ? tp_epoch_tag(epoch_ptr, a.layers_per_step, ag_layer, &abuf) : 0u;

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float g[8];
      ld_bf16x8(gamma + c, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * g[j];
      st_bf16x8(out + (long long)t * ldo + c, v[i]);
      // peers receive the same bf16 rounding as the local copy
      if (ag_layer >= 0) ag_put8(a, abuf, a.rank * a.rows + t, c, v[i]);
    }
  }
  if (ag_layer >= 0) ag_publish(a, abuf, atag, a.rank * a.rows + t);
}

// All-gather of this rank's rows x [rows, H] (bf16): one CTA per row.
__global__ void __launch_bounds__(256) tp_ag_send_kernel(TpArgs a, const int64_t* __restrict__ epoch_ptr, int layer,
                                                         const bf16* __restrict__ x, long long ldx, int rows) {
  griddep_wait();
  griddep_launch();
  int buf;
  const uint32_t tag = tp_epoch_tag(epoch_ptr, a.layers_per_step, layer, &buf);
  const int t = blockIdx.x;
  if (t >= rows) return;
  for (int c = threadIdx.x * 8; c < a.H; c += blockDim.x * 8) {
    float v[8];
    ld_bf16x8(x + (long long)t * ldx + c, v);
    ag_put8(a, buf, a.rank * a.rows + t, c, v);
  }
  ag_publish(a, buf, tag, a.rank * a.rows + t);
}

static void check_tp(const TpArgs& a) {
  if (a.world < 1 || a.world > 8 || a.rank < 0 || a.rank >= a.world) throw std::runtime_error("tp: bad world / rank");
  if (a.H % 8 || a.H > 8192) throw std::runtime_error("tp: hidden size must be a multiple of 8, at most 8192");
  if (a.layers_per_step < 2 || a.layers_per_step % 2) throw std::runtime_error("tp: layers per step must be even");
  for (int r = 0; r < a.world; ++r)
    if (!a.base[r] || (a.base[r] & 255)) throw std::runtime_error("tp: bad rank base pointer");
}

void tp_rs_add_rmsnorm(const TpArgs& a, const int64_t* epoch, int layer, int slots, void* residual, const void* gamma,
                       void* out, long long ldo, float eps, int ag_layer, long long budget, int* err, int rows,
                       cudaStream_t s) {
  check_tp(a);
  if (rows <= 0) return;
  if (rows > a.rows || slots < 1) throw std::runtime_error("tp: bad reduce-scatter rows / slots");
  launch_k(tp_rs_add_rmsnorm_kernel, dim3(rows), dim3(256), 0, s, a, epoch, layer, slots, static_cast<bf16*>(residual),
           static_cast<const bf16*>(gamma), static_cast<bf16*>(out), ldo, eps, ag_layer, budget, err);
}

void tp_ag_send(const TpArgs& a, const int64_t* epoch, int layer, const void* x, long long ldx, int rows,
                cudaStream_t s) {
  check_tp(a);
  if (rows <= 0) return;
  if (rows > a.rows) throw std::runtime_error("tp: more rows than a rank owns");
  launch_k(tp_ag_send_kernel, dim3(rows), dim3(256), 0, s, a, epoch, layer, static_cast<const bf16*>(x), ldx, rows);
}

}  // namespace sp
