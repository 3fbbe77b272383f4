// Block-scaled fp8 GEMM on the 5th-generation tensor cores (tcgen05.mma
// kind::f8f6f4 + TMEM), sm_100a.
//
//   D[m, n] = sum_kb sa(m, kb) * sb(n, kb) * sum_{k in block kb} Aq[m, k] * Bq[n, k]
//
// A is an e4m3 weight [rows, K] whose fp32 scales cover (sa_rows x 128) blocks
// (sa_rows = 128 for the 128x128 block format; 64 when a weight was re-laid out
// in 64-row halves, as the fused SwiGLU layout does); B is an e4m3 activation
// [N, K] with one fp32 scale per (row, 128 columns), stored K-block-major
// (sb[kb * ldsb + n]) so a tile's scales for one K block are contiguous.
//
// Promotion. The scales change every 128 columns of K, so one fp32 accumulator
// in TMEM cannot hold the sum. Per K block the MMA warp writes a fresh partial
// product into one of four TMEM buffers; eight epilogue warps (two per TMEM lane
// quarter, each owning half of the tile's columns) read it back with tcgen05.ld,
// multiply by sa * sb and add it into register accumulators while the tensor
// cores fill the next buffers (up to four K blocks ahead). The accumulation order over K blocks is fixed, so
// results are deterministic.
//
// Modes, as in the bf16 kernel: DENSE (persistent over (m, n) tiles), SPLITK
// (decode: the K blocks of one tile are split over independent CTAs that store
// fp32 partial slabs for the consumer), GROUPED (MoE experts: group g owns A rows
// [g*M, g*M+M) and a device-side range of sorted B rows; graph safe).
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer + TMEM
// owner, warps 2..9 = epilogue. Tiles: BLOCK_M 128, BLOCK_K 128 (one 128-byte
// swizzled row of fp8 per operand row), BLOCK_N in {32, 64, 128}.
//
// The reference declares the fp8 expert path only as an entry point of its
// resident decode stage (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/
// spark_resident_decode_stage.h:321-342, e4m3 weights with 128-block scales,
// launch :1053); the kernel is written here from scratch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ll.cuh"
#include "pdl.h"

namespace sp {

enum { F8_DENSE = 0, F8_SPLITK = 1, F8_GROUPED = 2 };
constexpr int F8_BM = 128;
constexpr int F8_BK = 128;
constexpr int F8_THREADS = 320;

struct Fp8KParams {
  int M, N, K;
  const float* sa;
  long long ldsa;
  int sa_rows, sa_blocks;
  const float* sb;
  long long ldsb;
  void* D;
  long long ldd;
  int trans_out, out_f32;
  int m_tiles, n_tiles, num_tiles, splits;
  const int* grp_rows;
  const int* grp_tiles;
  int num_groups;
  int a_evict_first, swiglu;
  float* ws;
  long long split_stride;
  int* err;
  int no_promote;  // diagnostic: accumulate every K block in TMEM unscaled (wrong values, streaming ceiling)
  int ep_on;       // grouped: rows go straight to their source ranks' combine slots
  EpCombDev ep;
};

template <int BN, int MODE>
struct F8Cfg {
  static constexpr int A_BYTES = F8_BM * F8_BK;
  static constexpr int B_BYTES = BN * F8_BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = MODE == F8_SPLITK ? 4 : (BN >= 128 ? 6 : 8);
  // TMEM partial buffers: the MMA may run NPB K blocks ahead of the promotion
  static constexpr int NPB = 4;
  static constexpr int TMEM_COLS = NPB * BN < 32 ? 32 : NPB * BN;
  static constexpr int HALF = BN / 2;                       // columns per epilogue warp
  static constexpr int XBUF_BYTES = 2 * 64 * 17 * 4;        // SwiGLU exchange (2 halves x 64 rows x 16 cols)
  static constexpr int SC = 16;                              // K blocks per staged scale chunk
  static constexpr int SCALE_BYTES = 2 * SC * (BN + 2) * 4;  // [2 chunks][SC][BN activation + 2 weight scales]
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + XBUF_BYTES + SCALE_BYTES;
};

// Named barrier 1 over the 256 epilogue threads that also ANDs a flag, so every
// epilogue thread takes the same path after a timeout.
SP_DEVI bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

struct F8Tile {
  int a_row, b_row;
  int m_base, n_base;
  int m_valid, n_valid;
};

template <int BN, int MODE>
SP_DEVI bool f8_tile(const Fp8KParams& p, int t, F8Tile& ti) {
  const int mt = t % p.m_tiles;
  const int q = t / p.m_tiles;
  if (MODE == F8_GROUPED) {
    int lo = 0, hi = p.num_groups;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(p.grp_tiles + mid) <= q) lo = mid; else hi = mid;
    }
    const int nt = q - __ldg(p.grp_tiles + lo);
    const int r0 = __ldg(p.grp_rows + lo), r1 = __ldg(p.grp_rows + lo + 1);
    ti.a_row = lo * p.M + mt * F8_BM;
    ti.b_row = r0 + nt * BN;
    ti.m_base = mt * F8_BM;
    ti.n_base = ti.b_row;
    ti.m_valid = min(F8_BM, p.M - mt * F8_BM);
    ti.n_valid = min(BN, r1 - ti.b_row);
    return ti.n_valid > 0;
  }
  const int nt = q % p.n_tiles;
  ti.a_row = mt * F8_BM;
  ti.b_row = nt * BN;
  ti.m_base = mt * F8_BM;
  ti.n_base = nt * BN;
  ti.m_valid = min(F8_BM, p.M - mt * F8_BM);
  ti.n_valid = min(BN, p.N - nt * BN);
  return true;
}

// Writes this thread's HALF accumulators of row m (columns c_lo ..) of a tile.
template <int BN>
SP_DEVI void f8_store_row(const Fp8KParams& p, void* Dp, long long ldd, int out_f32, int trans_out, const F8Tile& ti,
                          int m, int c_lo, const float* acc) {
  constexpr int HALF = BN / 2;
  if (m >= ti.m_valid) return;
  const long long mg = ti.m_base + m;
  if (out_f32) {
    float* D = reinterpret_cast<float*>(Dp);
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const int n = c_lo + j;
      if (n < ti.n_valid) {
        const long long ng = ti.n_base + n;
        if (trans_out) D[ng * ldd + mg] = acc[j];
        else D[mg * ldd + ng] = acc[j];
      }
    }
    return;
  }
  __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(Dp);
  if (trans_out) {
#pragma unroll
    for (int j = 0; j < HALF; ++j) {
      const int n = c_lo + j;
      if (n < ti.n_valid) D[(long long)(ti.n_base + n) * ldd + mg] = __float2bfloat16_rn(acc[j]);
    }
  } else {
    __nv_bfloat16* dst = D + mg * ldd + ti.n_base + c_lo;
    const bool vec = c_lo + HALF <= ti.n_valid && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (vec) {
#pragma unroll
      for (int j = 0; j < HALF; j += 8) st_bf16x8(dst + j, acc + j);
    } else {
#pragma unroll
      for (int j = 0; j < HALF; ++j)
        if (c_lo + j < ti.n_valid) dst[j] = __float2bfloat16_rn(acc[j]);
    }
  }
}

// Split-K CTAs with narrow tiles keep two per SM (registers capped at 102).
template <int BN, int MODE>
__global__ void __launch_bounds__(F8_THREADS, (MODE == F8_SPLITK && BN <= 32) ? 2 : 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const Fp8KParams p) {
  using C = F8Cfg<BN, MODE>;
  constexpr int HALF = C::HALF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* pfull = empty + C::STAGES;   // partial product of one K block ready (MMA -> epilogue)
  uint64_t* pempty = pfull + C::NPB;     // partial buffer read back (epilogue -> MMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pempty + C::NPB);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_ntiles = s_err + 1;
  float* xbuf = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);
  float* s_sb = xbuf + C::XBUF_BYTES / 4;            // [2][SC][BN]
  float* s_sa = s_sb + 2 * C::SC * BN;               // [2][SC][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < C::NPB; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], 256);
    }
    *s_err = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc<C::TMEM_COLS>(tmem_slot);
    tmem_relinquish();
    tc_fence_before();
  }
  const bool prefetch_a = (MODE != F8_GROUPED) && p.a_evict_first;
  const bool is_producer = (warp == 0 && lane == 0);
  if (MODE == F8_GROUPED) griddep_wait();
  if (threadIdx.x == 0) {
    int nt = p.num_tiles;
    if (MODE == F8_GROUPED) nt = p.m_tiles * __ldg(p.grp_tiles + p.num_groups);
    *s_ntiles = nt;
  }
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  if (!(prefetch_a && is_producer)) griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = *s_ntiles;

  int kb_begin = 0, kb_end = (p.K + F8_BK - 1) / F8_BK;
  int tile_first = blockIdx.x, tile_step = gridDim.x;
  int ks = 0;
  if (MODE == F8_SPLITK) {
    ks = blockIdx.x % p.splits;
    const int total = kb_end;
    kb_begin = (int)((long long)total * ks / p.splits);
    kb_end = (int)((long long)total * (ks + 1) / p.splits);
    tile_first = blockIdx.x / p.splits;
    tile_step = 1 << 30;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = p.a_evict_first ? policy_evict_first() : policy_evict_last();
      int it = 0, pre = 0;
      bool ok = true;
      if (prefetch_a) {
        if (tile_first < num_tiles) {
          F8Tile t0;
          f8_tile<BN, MODE>(p, tile_first, t0);
          pre = min(C::STAGES, kb_end - kb_begin);
          for (int j = 0; j < pre; ++j) {
            mbar_arrive_expect_tx(&full[j], C::STAGE_BYTES);
            tma_load_2d_hint(smem + j * C::STAGE_BYTES, &tmA, &full[j], (kb_begin + j) * F8_BK, t0.a_row, pol_a);
          }
        }
        griddep_wait();
      }
      for (int t = tile_first; t < num_tiles && ok; t += tile_step) {
        F8Tile ti;
        if (!f8_tile<BN, MODE>(p, t, ti)) continue;
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          if (it < pre) {
            tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], kb * F8_BK, ti.b_row);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1, s_err, p.err, kErrWaitTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d_hint(sa, &tmA, &full[s], kb * F8_BK, ti.a_row, pol_a);
          tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], kb * F8_BK, ti.b_row);
        }
      }
      if (!ok) {
        for (int j = 0; j < C::STAGES && j < it; ++j) {
          const int i2 = it - 1 - j;
          mbar_wait(&full[i2 % C::STAGES], (i2 / C::STAGES) & 1, s_err, nullptr, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(F8_BM, BN);
      int it = 0, tcount = 0;
      bool ok = true;
      const bool np = p.no_promote != 0;
      for (int t = tile_first; t < num_tiles && ok; t += tile_step) {
        F8Tile ti;
        if (!f8_tile<BN, MODE>(p, t, ti)) continue;
        if (np && !mbar_wait(&pempty[0], ((tcount & 1) ^ 1), s_err, p.err, kErrWaitTimeoutMma)) { ok = false; break; }
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          const int b = np ? 0 : it % C::NPB;
          const uint32_t bph = (it / C::NPB) & 1;
          if (!np && !mbar_wait(&pempty[b], bph ^ 1, s_err, p.err, kErrWaitTimeoutMma)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, s_err, p.err, kErrWaitTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t adesc = sdesc_kmajor_sw128(sa);
          const uint64_t bdesc = sdesc_kmajor_sw128(sa + C::A_BYTES);
          const uint32_t d_tmem = tmem_base + b * BN;
#pragma unroll
          for (int k = 0; k < F8_BK / 32; ++k)  // 32 fp8 of K = 32 bytes -> +2 in the start-address field
            umma_f8(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (k > 0 || (np && kb > kb_begin)) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (!np) umma_commit(&pfull[b]);
        }
        if (np && ok) umma_commit(&pfull[0]);
        ++tcount;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (promotion)
    const int ew = warp - 2;
    const int q = warp & 3;       // TMEM lane quarter
    const int h = ew >> 2;        // column half
    const int m = q * 32 + lane;  // tile row
    const int c_lo = h * HALF;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    // Scales are staged per chunk of SC K blocks in shared memory (double buffered):
    // the next chunk's global loads are in flight while this chunk is promoted, so no
    // K block waits on a scale load.
    constexpr int SC = C::SC;
    constexpr int NSB = (SC * BN + 255) / 256;  // activation-scale items per thread per chunk
    // K blocks promoted per TMEM round trip (narrow tiles). Two measured slower on the
    // Kimi-K2 decode shape (8-layer step 4.98 -> ~5.12 ms): waiting for a pair of partials
    // holds the first one back.
    constexpr int KBP = 1;
    const int etid = threadIdx.x - 64;
    const int my_sa = p.sa_rows == 64 ? (m >> 6) : 0;
    int it = 0, tcount = 0;
    bool ok = true;
    for (int t = tile_first; t < num_tiles && ok; t += tile_step) {
      F8Tile ti;
      if (!f8_tile<BN, MODE>(p, t, ti)) continue;
      float acc[HALF];
#pragma unroll
      for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
      if (p.no_promote) {
        if (!mbar_wait(&pfull[0], tcount & 1, s_err, p.err, kErrWaitTimeoutEpilogue)) { ok = false; }
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HALF; c += 16) {
            float v[16];
            tmem_ld16(lane_addr + c_lo + c, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[c + j] = v[j];
          }
          tc_fence_before();
          mbar_arrive(&pempty[0]);
        }
        ++tcount;
        ok = epi_bar_and(ok);
        if (!ok) break;
      }
      const int nkb = p.no_promote ? 0 : kb_end - kb_begin;
      const int nch = (nkb + SC - 1) / SC;
      const int blk0 = ti.a_row / p.sa_rows;
      float rsb[NSB], rsa = 0.f;
      auto load_chunk = [&](int ch) {
        const int kb0 = kb_begin + ch * SC;
#pragma unroll
        for (int u = 0; u < NSB; ++u) {
          const int i = etid + u * 256;
          const int j = i / BN, col = i - (i / BN) * BN;
          const int kb = kb0 + j;
          rsb[u] = (i < SC * BN && kb < kb_end && col < ti.n_valid)
                       ? __ldg(p.sb + (long long)kb * p.ldsb + ti.n_base + col) : 0.f;
        }
        if (etid < 2 * SC) {
          const int j = etid >> 1, r = etid & 1, kb = kb0 + j;
          const int blk = blk0 + r;
          rsa = (kb < kb_end && r * p.sa_rows < F8_BM && blk < p.sa_blocks) ? __ldg(p.sa + (long long)blk * p.ldsa + kb)
                                                                           : 0.f;
        }
      };
      auto store_chunk = [&](int ch) {
        float* dsb = s_sb + (ch & 1) * SC * BN;
#pragma unroll
        for (int u = 0; u < NSB; ++u) {
          const int i = etid + u * 256;
          if (i < SC * BN) dsb[i] = rsb[u];
        }
        if (etid < 2 * SC) s_sa[(ch & 1) * SC * 2 + etid] = rsa;
      };
      load_chunk(0);
      store_chunk(0);
      ok = epi_bar_and(ok);
      for (int ch = 0; ch < nch; ++ch) {
        if (ch + 1 < nch) load_chunk(ch + 1);
        const float* csb = s_sb + (ch & 1) * SC * BN + c_lo;
        const float* csa = s_sa + (ch & 1) * SC * 2 + my_sa;
        const int kend = min(SC, nkb - ch * SC);
        if constexpr (HALF > 32) {
          // wide tiles: one K block at a time, one 16-column TMEM load in registers at once
          for (int j = 0; j < kend; ++j, ++it) {
            if (!ok) continue;
            const int b = it % C::NPB;
            const uint32_t bph = (it / C::NPB) & 1;
            if (!mbar_wait(&pfull[b], bph, s_err, p.err, kErrWaitTimeoutEpilogue)) { ok = false; continue; }
            tc_fence_after();
            const float sa_v = m < ti.m_valid ? csa[j * 2] : 0.f;
#pragma unroll
            for (int c = 0; c < HALF; c += 16) {
              float v[16];
              tmem_ld16(lane_addr + b * BN + c_lo + c, v);
#pragma unroll
              for (int q4 = 0; q4 < 16; q4 += 4) {
                const float4 sb4 = *reinterpret_cast<const float4*>(csb + j * BN + c + q4);
                acc[c + q4] = fmaf(v[q4], sa_v * sb4.x, acc[c + q4]);
                acc[c + q4 + 1] = fmaf(v[q4 + 1], sa_v * sb4.y, acc[c + q4 + 1]);
                acc[c + q4 + 2] = fmaf(v[q4 + 2], sa_v * sb4.z, acc[c + q4 + 2]);
                acc[c + q4 + 3] = fmaf(v[q4 + 3], sa_v * sb4.w, acc[c + q4 + 3]);
              }
            }
            tc_fence_before();
            mbar_arrive(&pempty[b]);
          }
        } else {
          // K blocks in groups of KBP: every partial of a group is waited for, then all of
          // their TMEM loads are issued before one wait (one round trip per group)
          for (int j = 0; j < kend; j += KBP) {
            const int nk = min(KBP, kend - j);
            if (!ok) { it += nk; continue; }
            int bufs[KBP];
            bool got = true;
#pragma unroll
            for (int u = 0; u < KBP; ++u) {
              if (u >= nk) break;
              bufs[u] = (it + u) % C::NPB;
              if (got && !mbar_wait(&pfull[bufs[u]], ((it + u) / C::NPB) & 1, s_err, p.err, kErrWaitTimeoutEpilogue))
                got = false;
            }
            if (!got) { ok = false; it += nk; continue; }
            tc_fence_after();
            uint32_t r[KBP][HALF / 16][16];
#pragma unroll
            for (int u = 0; u < KBP; ++u) {
              if (u >= nk) break;
#pragma unroll
              for (int c = 0; c < HALF / 16; ++c) tmem_ld16_issue(lane_addr + bufs[u] * BN + c_lo + c * 16, r[u][c]);
            }
#pragma unroll
            for (int u = 0; u < KBP; ++u) {
              if (u >= nk) break;
#pragma unroll
              for (int c = 0; c < HALF / 16; ++c) tmem_ld_wait(r[u][c]);
            }
            tc_fence_before();
#pragma unroll
            for (int u = 0; u < KBP; ++u) {
              if (u >= nk) break;
              mbar_arrive(&pempty[bufs[u]]);  // the partials are in registers: release the buffers first
            }
#pragma unroll
            for (int u = 0; u < KBP; ++u) {
              if (u >= nk) break;
              const float sa_v = m < ti.m_valid ? csa[(j + u) * 2] : 0.f;
#pragma unroll
              for (int c = 0; c < HALF / 16; ++c) {
#pragma unroll
                for (int q4 = 0; q4 < 16; q4 += 4) {
                  const float4 sb4 = *reinterpret_cast<const float4*>(csb + (j + u) * BN + c * 16 + q4);
                  const int a0 = c * 16 + q4;
                  acc[a0] = fmaf(__uint_as_float(r[u][c][q4]), sa_v * sb4.x, acc[a0]);
                  acc[a0 + 1] = fmaf(__uint_as_float(r[u][c][q4 + 1]), sa_v * sb4.y, acc[a0 + 1]);
                  acc[a0 + 2] = fmaf(__uint_as_float(r[u][c][q4 + 2]), sa_v * sb4.z, acc[a0 + 2]);
                  acc[a0 + 3] = fmaf(__uint_as_float(r[u][c][q4 + 3]), sa_v * sb4.w, acc[a0 + 3]);
                }
              }
            }
            it += nk;
          }
        }
        if (ch + 1 < nch) store_chunk(ch + 1);
        ok = epi_bar_and(ok);
      }
      if (!ok) break;
      if (MODE == F8_SPLITK) {
        f8_store_row<BN>(p, p.ws + (size_t)ks * p.split_stride, p.trans_out ? p.M : p.N, 1, p.trans_out, ti, m, c_lo,
                         acc);
      } else if (MODE == F8_GROUPED && p.swiglu) {
        // rows [0, 64) of the tile are gate features, rows [64, 128) the matching up
        // features: exchange through shared memory, write silu(g) * u.
        __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(p.D);
        float* xb = xbuf + h * 64 * 17;
        const int f = (ti.m_base >> 1) + m;
#pragma unroll
        for (int c = 0; c < HALF; c += 16) {
          if (m >= 64) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[(m - 64) * 17 + j] = acc[c + j];
          }
          asm volatile("bar.sync 1, 256;" ::: "memory");
          if (m < 64 && 2 * m < ti.m_valid) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = c_lo + c + j;
              if (n < ti.n_valid) {
                const float g = acc[c + j], u = xb[m * 17 + j];
                D[(long long)(ti.n_base + n) * p.ldd + f] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
              }
            }
          }
          asm volatile("bar.sync 1, 256;" ::: "memory");
        }
      } else if (MODE == F8_GROUPED && p.ep_on) {
        int ebuf;
        const uint32_t etag = ep_comb_tag(p.ep, &ebuf);
#pragma unroll
        for (int j = 0; j < HALF; ++j)
          if (c_lo + j < ti.n_valid)
            ep_comb_store(p.ep, ebuf, etag, ti.n_base + c_lo + j, ti.m_base + m, acc[j], m < ti.m_valid);
      } else {
        f8_store_row<BN>(p, p.D, p.ldd, p.out_f32, p.trans_out, ti, m, c_lo, acc);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<C::TMEM_COLS>(tmem_base);
  }
}

// ======================================================================= host

template <int BN, int MODE>
static void launch_fp8(const Fp8Launch& g, Fp8KParams& p) {
  using C = F8Cfg<BN, MODE>;
  CUtensorMap ta, tb;
  make_tmap_2d(&ta, g.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.a_rows, g.K, g.lda, F8_BM, F8_BK);
  make_tmap_2d(&tb, g.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.b_rows, g.K, g.ldb, BN, F8_BK);
  auto kern = gemm_fp8_kernel<BN, MODE>;
  set_smem_bytes(kern, C::SMEM_BYTES);
  prefer_max_smem_carveout(reinterpret_cast<const void*>(kern));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attrs[1];
  cfg.blockDim = dim3(F8_THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = g.stream;
  int grid;
  if (MODE == F8_SPLITK) grid = p.num_tiles * p.splits;
  else if (MODE == F8_GROUPED) grid = g.num_sms;
  else grid = std::min(p.num_tiles, g.num_sms);
  cfg.gridDim = dim3(std::max(grid, 1), 1, 1);
  cfg.attrs = attrs;
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("fp8 gemm launch failed: ") + cudaGetErrorString(e));
}

template <int MODE>
static void fp8_dispatch_bn(int bn, const Fp8Launch& g, Fp8KParams& p) {
  switch (bn) {
    case 32: launch_fp8<32, MODE>(g, p); break;
    case 64: launch_fp8<64, MODE>(g, p); break;
    case 128: launch_fp8<128, MODE>(g, p); break;
    default: throw std::runtime_error("gemm_fp8: BLOCK_N must be 32, 64 or 128");
  }
}

int gemm_fp8(const Fp8Launch& g) {
  if (g.M <= 0 || g.N <= 0) return 0;
  if (g.K <= 0 || g.K % F8_BK != 0) throw std::runtime_error("gemm_fp8: K must be a positive multiple of 128");
  if (g.sa_rows != 64 && g.sa_rows != 128) throw std::runtime_error("gemm_fp8: weight scale blocks are 64 or 128 rows");
  if (!g.sa || !g.sb) throw std::runtime_error("gemm_fp8: scales missing");
  Fp8KParams p = {};
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.sa = g.sa; p.ldsa = g.ldsa; p.sa_rows = g.sa_rows; p.sa_blocks = g.sa_blocks;
  p.sb = g.sb; p.ldsb = g.ldsb;
  p.D = g.D; p.ldd = g.ldd; p.trans_out = g.trans_out; p.out_f32 = g.out_f32;
  p.err = g.err;
  p.a_evict_first = g.a_evict_first;
  p.swiglu = g.swiglu;
  static const int no_promote = [] {  // diagnostic only: SPARKPIPE_FP8_NOPROMOTE=1 gives wrong values
    const char* e = std::getenv("SPARKPIPE_FP8_NOPROMOTE");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  p.no_promote = no_promote;
  if (g.swiglu && (!g.grouped || !g.trans_out || g.out_f32 || g.M % 128 != 0))
    throw std::runtime_error("gemm_fp8: fused SwiGLU needs a grouped, transposed bf16 GEMM with M % 128 == 0");
  p.m_tiles = (g.M + F8_BM - 1) / F8_BM;
  if (g.ep) {
    if (!g.grouped || !g.trans_out || g.out_f32 || g.swiglu || g.M != g.ep->H || g.ep->H % 2)
      throw std::runtime_error("gemm_fp8: the combine epilogue needs a grouped, transposed bf16 GEMM with M = hidden");
    p.ep_on = 1;
    const EpComb& e = *g.ep;
    for (int r = 0; r < 8; ++r) p.ep.base[r] = e.base[r];
    p.ep.comb_off = e.comb_off; p.ep.cap = e.cap; p.ep.kk = e.kk; p.ep.H = e.H;
    p.ep.layers_per_step = e.layers_per_step; p.ep.comb_dst = e.comb_dst; p.ep.epoch = e.epoch; p.ep.layer = e.layer;
  }
  if (g.grouped) {
    if (g.M % g.sa_rows != 0) throw std::runtime_error("gemm_fp8: grouped M must be a multiple of the scale block");
    const int bn = g.block_n > 0 ? g.block_n : 32;
    p.grp_rows = g.grp_rows;
    p.grp_tiles = g.grp_tiles;
    p.num_groups = g.num_groups;
    fp8_dispatch_bn<F8_GROUPED>(bn, g, p);
    return 1;
  }
  const int bn = g.block_n > 0 ? g.block_n : (g.N <= 32 ? 32 : (g.N <= 64 ? 64 : 128));
  p.n_tiles = (g.N + bn - 1) / bn;
  p.num_tiles = p.m_tiles * p.n_tiles;
  const int kbs = g.K / F8_BK;
  int splits = g.splits;
  if (splits <= 0) {
    // the most splits that keep one CTA per SM, at least two K blocks each (as the bf16 GEMM)
    splits = std::max(1, std::min({g.num_sms / std::max(1, p.num_tiles), kbs / 2, 16}));
  }
  if (splits > kbs) splits = kbs;
  const long long slab = (long long)g.M * g.N;
  const int out_cols = g.trans_out ? g.M : g.N;
  if (splits > 1 && (!g.ws || slab * splits > g.ws_floats || out_cols % 4 != 0 ||
                     (!g.slab_out && (g.ldd % 4 != 0 || (reinterpret_cast<uintptr_t>(g.D) & 15) != 0))))
    splits = 1;
  p.ws = g.ws;
  p.split_stride = slab;
  p.splits = splits;
  if (splits > 1) {
    fp8_dispatch_bn<F8_SPLITK>(bn, g, p);
    if (g.slab_out) return -splits;
    const int rows = g.trans_out ? g.N : g.M;
    const int cols = g.trans_out ? g.M : g.N;
    split_reduce(g.ws, slab, splits, rows, cols, g.D, g.ldd, g.out_f32, g.stream);
    return 2;
  }
  fp8_dispatch_bn<F8_DENSE>(bn, g, p);
  return 1;
}

// ------------------------------------------------------------------ activation quant
// One warp per (row, 128-column block): amax -> scale = amax / 448 -> e4m3 values.
// Row r reads source row src_idx[r] / idx_div when a gather index is given (the
// MoE expert-sorted layout); scales are written K-block-major: s[kb * lds + r].
// With `rows_dev` the live row count is read from device memory (rows beyond it
// are skipped; `rows` is then the capacity); warps stride over the work.
__global__ void quant_act_fp8_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                     const int* __restrict__ src_idx, int idx_div, const int* __restrict__ rows_dev,
                                     __nv_fp8_e4m3* __restrict__ q, long long ldq, float* __restrict__ s,
                                     long long lds, int rows, int cols) {
  griddep_wait();
  griddep_launch();
  const int nb = cols / 128;
  const int lane = threadIdx.x & 31;
  const int live = rows_dev ? min(rows, __ldg(rows_dev)) : rows;
  const long long total = (long long)live * nb;
  const long long wstep = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += wstep) {
    const int r = (int)(w / nb), b = (int)(w - (long long)r * nb);
    const long long src_row = src_idx ? (long long)(__ldg(src_idx + r) / idx_div) : (long long)r;
    const __nv_bfloat16* src = x + src_row * ldx + b * 128 + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f0 = __bfloat1622float2(hv[0]), f1 = __bfloat1622float2(hv[1]);
    float scale;
    const uint32_t o = warp_quant_e4m3_block(f0.x, f0.y, f1.x, f1.y, scale);
    *reinterpret_cast<uint32_t*>(q + (long long)r * ldq + b * 128 + lane * 4) = o;
    if (lane == 0) s[(long long)b * lds + r] = scale;
  }
}

void quant_act_fp8(const void* x, long long ldx, const int* src_idx, int idx_div, const int* rows_dev, void* q,
                   long long ldq, float* s, long long lds, int rows, int cols, int num_sms, cudaStream_t st) {
  if (rows <= 0) return;
  if (cols % 128 != 0) throw std::runtime_error("quant_act_fp8: cols % 128");
  if ((reinterpret_cast<uintptr_t>(x) & 7) || (ldx & 3)) throw std::runtime_error("quant_act_fp8: x not 8B aligned");
  const long long n = (long long)rows * (cols / 128);
  const int warps = 8;
  const long long want = (n + warps - 1) / warps;
  const long long cap = (long long)num_sms * 8;  // 8 CTAs of 8 warps per SM; warps stride beyond that
  launch_k(quant_act_fp8_kernel, dim3((unsigned)std::min(want, cap)), dim3(warps * 32), 0, st,
           (const __nv_bfloat16*)x, ldx, src_idx, idx_div < 1 ? 1 : idx_div, rows_dev, (__nv_fp8_e4m3*)q, ldq, s,
           lds, rows, cols);
}

// ------------------------------------------------------------------ weight init / quant
// Counter-based normal samples: a 64-bit mix (splitmix64 finaliser) of (seed,
// index) gives two uniforms, Box-Muller turns them into two N(0, 1) values.
SP_DEVI uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
SP_DEVI float2 normal2(uint64_t seed, uint64_t i) {
  const uint64_t r = mix64(seed * 0x9e3779b97f4a7c15ull + i);
  const float u1 = (float(uint32_t(r >> 40)) + 1.f) * (1.f / 16777217.f);  // (0, 1]
  const float u2 = float(uint32_t(r & 0xffffffu)) * (1.f / 16777216.f);
  const float rad = sqrtf(-2.f * __logf(u1));
  float sn, cs;
  __sincosf(6.283185307f * u2, &sn, &cs);
  return make_float2(rad * cs, rad * sn);
}

// One CTA (256 threads) per 128x128 block of a [rows, cols] e4m3 weight; each
// thread holds an 8 x 8 patch (64 values) in registers, the block amax gives the
// fp32 scale amax / 448. Source: `src` (bf16, pitch cols) when given, otherwise
// seeded N(0, std) samples at flat index flat0 + row * cols + col, so any shard of
// a weight is reproducible on its own.
__global__ void __launch_bounds__(256) quant_weight_fp8_kernel(const __nv_bfloat16* __restrict__ src,
                                                               uint64_t seed, long long flat0, float std_,
                                                               __nv_fp8_e4m3* __restrict__ q, float* __restrict__ s,
                                                               int rows, int cols) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[8];
  const int nbc = cols / 128;
  const int br = blockIdx.x / nbc, bc = blockIdx.x - (blockIdx.x / nbc) * nbc;
  const int tid = threadIdx.x;
  // thread -> 8 rows x 8 columns: column group tid % 16 (8 columns), row group tid / 16 (8 rows)
  const int c0 = bc * 128 + (tid & 15) * 8;
  const int rg = (tid >> 4) * 8;
  float v[64];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = br * 128 + rg + i;
    if (r < rows) {
      if (src) {
        ld_bf16x8(src + (long long)r * cols + c0, v + i * 8);
      } else {
        const long long base = flat0 + (long long)r * cols + c0;
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          const float2 z = normal2(seed, (uint64_t)(base + j) >> 1);
          v[i * 8 + j] = z.x * std_;
          v[i * 8 + j + 1] = z.y * std_;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i * 8 + j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i * 8 + j]));
  }
  amax = warp_max(amax);
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / scale;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = br * 128 + rg + i;
    if (r < rows) {
      __nv_fp8x4_e4m3 a(make_float4(v[i * 8] * inv, v[i * 8 + 1] * inv, v[i * 8 + 2] * inv, v[i * 8 + 3] * inv));
      __nv_fp8x4_e4m3 b(make_float4(v[i * 8 + 4] * inv, v[i * 8 + 5] * inv, v[i * 8 + 6] * inv, v[i * 8 + 7] * inv));
      uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
      *reinterpret_cast<uint2*>(q + (long long)r * cols + c0) = packed;
    }
  }
  if (tid == 0) s[(long long)br * nbc + bc] = scale;
}

void quant_weight_fp8(const void* src, uint64_t seed, long long flat0, float std_, void* q, float* s, int rows,
                      int cols, cudaStream_t st) {
  if (rows <= 0) return;
  if (cols % 128 != 0) throw std::runtime_error("quant_weight_fp8: cols % 128");
  if (flat0 % 2 != 0) throw std::runtime_error("quant_weight_fp8: flat0 must be even (samples come in pairs)");
  const long long nblk = (long long)((rows + 127) / 128) * (cols / 128);
  launch_k(quant_weight_fp8_kernel, dim3((unsigned)nblk), dim3(256), 0, st, (const __nv_bfloat16*)src, seed, flat0,
           std_, (__nv_fp8_e4m3*)q, s, rows, cols);
}

void kernel_attrs_fp8(std::vector<KernelAttr>& out) {
#define SP_F8_ATTR(BN, MODE) push_kernel_attr(out, "gemm_fp8_kernel<" #BN "," #MODE ">", gemm_fp8_kernel<BN, MODE>)
  SP_F8_ATTR(32, 0); SP_F8_ATTR(64, 0); SP_F8_ATTR(128, 0);
  SP_F8_ATTR(32, 1); SP_F8_ATTR(64, 1); SP_F8_ATTR(128, 1);
  SP_F8_ATTR(32, 2); SP_F8_ATTR(64, 2); SP_F8_ATTR(128, 2);
#undef SP_F8_ATTR
}

}  // namespace sp
