// NVFP4 weight storage for sm_100a: 4-bit E2M1 values in 16-element blocks, one
// FP8 E4M3 scale per block and one FP32 scale per tensor
// (x = e2m1 * e4m3_block_scale * tensor_scale). Two values per byte, element 2i in
// the low nibble. This file expands NVFP4 rows to bf16: one thread per 16-element
// block (8 packed bytes in, 32 bf16 bytes out, both 16-byte aligned), so a row of K
// elements is K/16 independent threads and the kernel runs at copy bandwidth.
//
// Reference: the NVFP4 expert path named in crates/spark-abi/vendor/sparkpipe (b12x
// packs, QUANTIZATION_NVFP4_4BIT in crates/spark-node/src/rank_daemon/ring_runtime.rs:85);
// the format is the published NVFP4 layout, the kernel is this framework's own.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "pdl.h"

namespace sp {

namespace {
// E2M1 nibble -> float from the format's fields, no table: bit 3 sign, bits 2..1
// exponent (bias 1), bit 0 mantissa. Exponent 0 is the subnormal 0 / 0.5; otherwise
// (1 + m/2) * 2^(e-1), whose fp32 pattern is exponent e + 126 and mantissa bit 22.
// (A __constant__ table indexed per lane serialises on the constant cache.)
SP_DEVI float e2m1_to_float(uint32_t code) {
  const uint32_t e = (code >> 1) & 3u, m = code & 1u;
  const float mag = e ? __uint_as_float(((e + 126u) << 23) | (m << 22)) : (m ? 0.5f : 0.f);
  return (code & 8u) ? -mag : mag;
}
}  // namespace

__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                     float tensor_scale, long long blocks, __nv_bfloat16* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  const uint2 q = reinterpret_cast<const uint2*>(packed)[b];
  __nv_fp8_e4m3 s8;
  s8.__x = scales[b];
  const float s = float(s8) * tensor_scale;
  // The block's 16 values share one scale, so the 8 scaled magnitudes are rounded to
  // bf16 once and kept as a 16-byte table in two 64-bit registers; each value is then a
  // shift out of the table plus the sign bit (bf16 rounding is symmetric, so
  // -round(m * s) == round(-m * s)).
  uint64_t lo = 0, hi = 0;
#pragma unroll
  for (uint32_t k = 0; k < 4; ++k) {
    lo |= uint64_t(__bfloat16_as_ushort(__float2bfloat16(e2m1_to_float(k) * s))) << (16 * k);
    hi |= uint64_t(__bfloat16_as_ushort(__float2bfloat16(e2m1_to_float(k + 4) * s))) << (16 * k);
  }
  auto bits = [&](uint32_t c) -> uint32_t {
    const uint64_t t = (c & 4u) ? hi : lo;
    return (uint32_t(t >> ((c & 3u) * 16u)) & 0xffffu) | ((c & 8u) << 12);
  };
  const uint32_t words[2] = {q.x, q.y};
  __align__(16) uint32_t v[8];
#pragma unroll
  for (int w = 0; w < 2; ++w)
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const uint32_t pair = words[w] >> (8 * n);
      v[w * 4 + n] = bits(pair & 0xfu) | (bits((pair >> 4) & 0xfu) << 16);
    }
  uint4* o = reinterpret_cast<uint4*>(out + b * 16);
  o[0] = reinterpret_cast<const uint4*>(v)[0];
  o[1] = reinterpret_cast<const uint4*>(v)[1];
}

void dequant_nvfp4(const uint8_t* packed, const uint8_t* scales, float tensor_scale, long long elements, void* out,
                   cudaStream_t s) {
  if (elements <= 0) return;
  if (elements % 16) throw std::runtime_error("dequant_nvfp4: element count must be a multiple of 16");
  const long long blocks = elements / 16;
  launch_k(dequant_nvfp4_kernel, dim3((unsigned)((blocks + 255) / 256)), dim3(256), 0, s, packed, scales, tensor_scale,
           blocks, reinterpret_cast<__nv_bfloat16*>(out));
}

}  // namespace sp
