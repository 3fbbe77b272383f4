// RMSNorm (+ fused residual add), MLA latent-KV write (latent RMSNorm + RoPE on
// the shared rope key + paged-cache store), query RoPE, and fp8 block quant.
//
// These are the ATTENTION_NORM / POST_ATTENTION_NORM / ROPE_KV_WRITE phases of
// the reference's resident decode stage
// (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:445-460,
// capability FUSED_ROPE_KV_WRITE :212) and its in-kernel activation quant
// (IN_KERNEL_INPUT_QUANT :310). All are HBM-bandwidth kernels: 16-byte
// vector loads, one warp per row, fp32 math.
//
// RoPE convention used across this package: adjacent pairs (x[2i], x[2i+1])
// rotate by angle_i; cos_sin[pos] holds rope/2 cosines then rope/2 sines.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

using bf16 = __nv_bfloat16;

// One CTA (256 threads) per row; the row stays in registers (hidden <= 8192).
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const bf16* __restrict__ x, long long ldx,
                                                          bf16* __restrict__ res, const bf16* __restrict__ w,
                                                          bf16* __restrict__ out, long long ldo, int rows, int H,
                                                          float eps) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const bf16* xr = x + (long long)row * ldx;
  bf16* rr = res ? res + (long long)row * H : nullptr;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      ld_bf16x8(xr + c, v[i]);
      if (rr) {
        float r[8];
        ld_bf16x8(rr + c, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(v[i][j] + r[j]));
        st_bf16x8(rr + c, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float part[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float inv = rsqrtf(tot / H + eps);
  bf16* orow = out + (long long)row * ldo;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float g[8];
      ld_bf16x8(w + c, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * g[j];
      st_bf16x8(orow + c, v[i]);
    }
  }
}

void add_rmsnorm(const void* x, long long ldx, void* residual, const void* w, void* out, long long ldo, int rows,
                 int hidden, float eps, cudaStream_t s) {
  if (rows <= 0) return;
  if (hidden % 8 != 0 || ldx % 8 != 0 || ldo % 8 != 0) throw std::runtime_error("add_rmsnorm: hidden/pitch % 8");
  if (hidden > 8192) throw std::runtime_error("add_rmsnorm: hidden <= 8192");
  launch_k(add_rmsnorm_kernel, dim3(rows), dim3(256), 0, s, (const bf16*)x, ldx, (bf16*)residual, (const bf16*)w,
           (bf16*)out, ldo, rows, hidden, eps);
}

// Residual add + RMSNorm whose input is the sum of `splits` fp32 split-K slabs
// (x[t] = sum_s slab[s][t]): the split reduction of the producing GEMM fused
// into its consumer. One CTA (256 threads) per row, hidden <= 8192.
__global__ void __launch_bounds__(256) slab_add_rmsnorm_kernel(const float* __restrict__ slab, long long stride,
                                                               int splits, bf16* __restrict__ res,
                                                               const bf16* __restrict__ w, bf16* __restrict__ out,
                                                               long long ldo, int H, float eps) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  bf16* rr = res + (long long)row * H;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      const float* src = slab + (long long)row * H + c;
      float4 a = __ldcg(reinterpret_cast<const float4*>(src));
      float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
      for (int s2 = 1; s2 < splits; ++s2) {
        const float4 a2 = __ldcg(reinterpret_cast<const float4*>(src + s2 * stride));
        const float4 b2 = __ldcg(reinterpret_cast<const float4*>(src + s2 * stride + 4));
        a.x += a2.x; a.y += a2.y; a.z += a2.z; a.w += a2.w;
        b.x += b2.x; b.y += b2.y; b.z += b2.z; b.w += b2.w;
      }
      // the GEMM output is rounded to bf16 before the residual add, as in the unfused path
      const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
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
  __shared__ float part[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float inv = rsqrtf(tot / H + eps);
  bf16* orow = out + (long long)row * ldo;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c < H) {
      float g[8];
      ld_bf16x8(w + c, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * g[j];
      st_bf16x8(orow + c, v[i]);
    }
  }
}

void slab_add_rmsnorm(const float* slab, long long stride, int splits, void* residual, const void* w, void* out,
                      long long ldo, int rows, int hidden, float eps, cudaStream_t s) {
  if (rows <= 0) return;
  if (hidden % 8 != 0 || hidden > 8192) throw std::runtime_error("slab_add_rmsnorm: hidden % 8, <= 8192");
  launch_k(slab_add_rmsnorm_kernel, dim3(rows), dim3(256), 0, s, slab, stride, splits, (bf16*)residual,
           (const bf16*)w, (bf16*)out, ldo, hidden, eps);
}

// Decode prologue of MLA attention, one CTA (8 warps) per token. The token's
// q/kv projection row is either bf16 (`src`) or the sum of fp32 split-K slabs.
//   warp 0        : latent RMSNorm + RoPE on the rope key -> paged cache slot
//   all warps     : per head, q_nope -> q_nope_out[t, h, :] (bf16, compact) and
//                   RoPE(q_pe) -> q_lat[t, h, kv_lora:]
__global__ void __launch_bounds__(256) mla_decode_prep_kernel(
    const float* __restrict__ slab, long long stride, int splits, const bf16* __restrict__ src, long long lds,
    const bf16* __restrict__ nw, const int* __restrict__ pos, const float* __restrict__ cs,
    const int* __restrict__ slots, bf16* __restrict__ cache, bf16* __restrict__ q_nope_out,
    bf16* __restrict__ q_lat, int H, int dn, int dr, int L, int qoff, int kvoff, int row_len, float eps) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto val = [&](int c) -> float {
    if (slab) {
      const float* p = slab + (long long)t * row_len + c;
      float a = __ldcg(p);
      for (int s2 = 1; s2 < splits; ++s2) a += __ldcg(p + s2 * stride);
      return __bfloat162float(__float2bfloat16_rn(a));
    }
    return __bfloat162float(src[(long long)t * lds + c]);
  };
  const int p = pos[t];
  const float* cp = cs + (long long)p * dr;
  const int W = L + dr;
  if (warp == 0) {
    float v[32];
    float ss = 0.f;
    const int per = L / 32;  // <= 32
    for (int i = 0; i < per; ++i) {
      v[i] = val(kvoff + lane + i * 32);
      ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / L + eps);
    const int slot = slots[t];
    if (slot >= 0) {
      bf16* crow = cache + (long long)slot * W;
      for (int i = 0; i < per; ++i) {
        const int c = lane + i * 32;
        crow[c] = __float2bfloat16_rn(v[i] * inv * __bfloat162float(nw[c]));
      }
      for (int i = lane; i < dr / 2; i += 32) {
        const float x0 = val(kvoff + L + 2 * i), x1 = val(kvoff + L + 2 * i + 1);
        const float c = cp[i], sn = cp[dr / 2 + i];
        crow[L + 2 * i] = __float2bfloat16_rn(x0 * c - x1 * sn);
        crow[L + 2 * i + 1] = __float2bfloat16_rn(x0 * sn + x1 * c);
      }
    }
  }
  for (int h = warp; h < H; h += 8) {
    const int base = qoff + h * (dn + dr);
    bf16* qn = q_nope_out + ((long long)t * H + h) * dn;
    for (int c = lane; c < dn; c += 32) qn[c] = __float2bfloat16_rn(val(base + c));
    bf16* ql = q_lat + ((long long)t * H + h) * W + L;
    for (int i = lane; i < dr / 2; i += 32) {
      const float x0 = val(base + dn + 2 * i), x1 = val(base + dn + 2 * i + 1);
      const float c = cp[i], sn = cp[dr / 2 + i];
      ql[2 * i] = __float2bfloat16_rn(x0 * c - x1 * sn);
      ql[2 * i + 1] = __float2bfloat16_rn(x0 * sn + x1 * c);
    }
  }
}

void mla_decode_prep(const float* slab, long long stride, int splits, const void* src, long long lds,
                     const void* norm_w, const int* positions, const float* cos_sin, const int* slot_mapping,
                     void* cache, void* q_nope_out, void* q_lat, int T, int H, int dn, int dr, int kv_lora,
                     int q_off, int kv_off, int row_len, float eps, cudaStream_t s) {
  if (T <= 0) return;
  if (kv_lora % 32 != 0 || kv_lora > 1024) throw std::runtime_error("mla_decode_prep: kv_lora % 32, <= 1024");
  launch_k(mla_decode_prep_kernel, dim3(T), dim3(256), 0, s, slab, stride, splits, (const bf16*)src, lds,
           (const bf16*)norm_w, positions, cos_sin, slot_mapping, (bf16*)cache, (bf16*)q_nope_out, (bf16*)q_lat, H,
           dn, dr, kv_lora, q_off, kv_off, row_len, eps);
}

__global__ void mla_kv_write_kernel(const bf16* __restrict__ kv, long long ldkv, const bf16* __restrict__ nw,
                                    const int* __restrict__ pos, const float* __restrict__ cs,
                                    const int* __restrict__ slots, bf16* __restrict__ cache, bf16* __restrict__ lat,
                                    long long ldl, int T, int L, int R, float eps) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const bf16* src = kv + (long long)t * ldkv;
  constexpr int MAXV = 4;  // latent up to 1024 elements
  float v[MAXV][8];
  float ss = 0.f;
  int nv = 0;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane * 8 + i * 256;
    if (c < L) {
      ld_bf16x8(src + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
      nv = i + 1;
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / L + eps);
  const int slot = slots ? slots[t] : -1;
  const int W = L + R;
  bf16* crow = slot >= 0 ? cache + (long long)slot * W : nullptr;
  bf16* lrow = lat ? lat + (long long)t * ldl : nullptr;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (i < nv) {
      const int c = lane * 8 + i * 256;
      float g[8];
      ld_bf16x8(nw + c, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * g[j];
      if (crow) st_bf16x8(crow + c, v[i]);
      if (lrow) st_bf16x8(lrow + c, v[i]);
    }
  }
  const int p = pos[t];
  const float* cp = cs + (long long)p * R;
  for (int i = lane; i < R / 2; i += 32) {
    const float x0 = __bfloat162float(src[L + 2 * i]);
    const float x1 = __bfloat162float(src[L + 2 * i + 1]);
    const float c = cp[i], sn = cp[R / 2 + i];
    const bf16 y0 = __float2bfloat16_rn(x0 * c - x1 * sn);
    const bf16 y1 = __float2bfloat16_rn(x0 * sn + x1 * c);
    if (crow) { crow[L + 2 * i] = y0; crow[L + 2 * i + 1] = y1; }
    if (lrow) { lrow[L + 2 * i] = y0; lrow[L + 2 * i + 1] = y1; }
  }
}

void mla_kv_write(const void* kv, long long ldkv, const void* norm_w, const int* positions, const float* cos_sin,
                  const int* slot_mapping, void* cache, void* latent_out, long long ldl, int T, int kv_lora, int rope,
                  float eps, cudaStream_t s) {
  if (T <= 0) return;
  if (kv_lora % 256 != 0 || kv_lora > 1024) throw std::runtime_error("mla_kv_write: kv_lora must be 256..1024");
  const int warps = 8;
  launch_k(mla_kv_write_kernel, dim3((T + warps - 1) / warps), dim3(warps * 32), 0, s, (const bf16*)kv, ldkv,
           (const bf16*)norm_w, positions, cos_sin, slot_mapping, (bf16*)cache, (bf16*)latent_out, ldl, T, kv_lora,
           rope, eps);
}

__global__ void rope_q_kernel(const bf16* src, long long st, long long sh, int so, bf16* dst, long long dt,
                              long long dh, int doff, const int* __restrict__ pos, const float* __restrict__ cs, int T,
                              int H, int R) {
  griddep_wait();
  griddep_launch();
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * H) return;
  const int t = w / H, h = w % H;
  const bf16* s = src + t * st + h * sh + so;
  bf16* d = dst + t * dt + h * dh + doff;
  const float* cp = cs + (long long)pos[t] * R;
  for (int i = lane; i < R / 2; i += 32) {
    const float x0 = __bfloat162float(s[2 * i]);
    const float x1 = __bfloat162float(s[2 * i + 1]);
    const float c = cp[i], sn = cp[R / 2 + i];
    d[2 * i] = __float2bfloat16_rn(x0 * c - x1 * sn);
    d[2 * i + 1] = __float2bfloat16_rn(x0 * sn + x1 * c);
  }
}

void rope_q(const void* src, long long src_tok, long long src_head, int src_off, void* dst, long long dst_tok,
            long long dst_head, int dst_off, const int* positions, const float* cos_sin, int T, int H, int rope,
            cudaStream_t s) {
  if (T <= 0) return;
  const int warps = 8;
  const int n = T * H;
  launch_k(rope_q_kernel, dim3((n + warps - 1) / warps), dim3(warps * 32), 0, s, (const bf16*)src, src_tok, src_head,
           src_off, (bf16*)dst, dst_tok, dst_head, dst_off, positions, cos_sin, T, H, rope);
}

__global__ void quant_fp8_block_kernel(const bf16* __restrict__ x, long long ldx, __nv_fp8_e4m3* __restrict__ q,
                                       float* __restrict__ scales, int rows, int cols) {
  griddep_wait();
  griddep_launch();
  const int nb = cols / 128;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * nb) return;
  const int r = w / nb, b = w % nb;
  const bf16* src = x + (long long)r * ldx + b * 128 + lane * 4;
  float v[4];
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(src);
  float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* dst = q + (long long)r * cols + b * 128 + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[j] = __nv_fp8_e4m3(v[j] * inv);
  if (lane == 0) scales[(long long)r * nb + b] = scale;
}

void quant_fp8_block(const void* x, long long ldx, void* q, float* scales, int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  if (cols % 128 != 0) throw std::runtime_error("quant_fp8_block: cols % 128");
  const int n = rows * (cols / 128);
  const int warps = 8;
  launch_k(quant_fp8_block_kernel, dim3((n + warps - 1) / warps), dim3(warps * 32), 0, s, (const bf16*)x, ldx,
           (__nv_fp8_e4m3*)q, scales, rows, cols);
}

}  // namespace sp
