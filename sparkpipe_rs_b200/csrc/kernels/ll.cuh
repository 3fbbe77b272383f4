// Low-latency (LL) tagged words for peer-memory collectives, sm_100a.
//
// A 64-bit word carries 32 payload bits and a 32-bit tag (the collective's epoch
// + 1). A writer stores payload and tag together with one 64-bit store, which a
// reader observes whole, so seeing the current tag proves the payload arrived:
// no fences or flags are needed between peers. Every poll is bounded twice: by
// its own clock64 budget, and by the device status word (once any poll of the
// device gave up, the others give up at their next check), so a missing peer
// ends a kernel with kErrWaitTimeoutPeer instead of hanging it.
#pragma once

#include "common.cuh"

namespace sp {

using u64 = unsigned long long;

SP_DEVI u64 ll_word(uint32_t payload, uint32_t tag) { return (u64(tag) << 32) | payload; }
SP_DEVI void st_ll(u64* p, u64 w) { asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory"); }
SP_DEVI void st_ll2(u64* p, u64 a, u64 b) {  // two independent 64-bit elements (each single-copy atomic)
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
SP_DEVI u64 ld_ll(const u64* p) {
  u64 v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
SP_DEVI void ld_ll2(const u64* p, u64& a, u64& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
SP_DEVI uint32_t tag_of(u64 w) { return uint32_t(w >> 32); }

// Every poll is bounded twice: by its own clock64 budget, and by the device
// status word: once any poll of the device has given up (status set), every
// other poll gives up at its next check, so a kernel whose peer is gone ends
// after one budget, not one budget per word.
SP_DEVI bool poll_abort(const int* gerr) { return *reinterpret_cast<const volatile int*>(gerr) != 0; }

// Bounded poll of one word; returns its payload (0 and ok = false on timeout).
SP_DEVI uint32_t poll_ll(const u64* p, uint32_t tag, long long budget, bool& ok, int* gerr) {
  u64 w = ld_ll(p);
  if (tag_of(w) == tag) return uint32_t(w);
  const long long t0 = clock64();
  for (unsigned it = 1;; ++it) {
    w = ld_ll(p);
    if (tag_of(w) == tag) return uint32_t(w);
    if (clock64() - t0 > budget) { atomicCAS(gerr, 0, kErrWaitTimeoutPeer); ok = false; return 0; }
    if ((it & 255) == 0 && poll_abort(gerr)) { ok = false; return 0; }
  }
}
// Bounded poll of four consecutive words (8 bf16); false on timeout.
SP_DEVI bool poll_ll4(const u64* p, uint32_t tag, long long budget, uint32_t (&v)[4], int* gerr) {
  u64 w0, w1, w2, w3;
  ld_ll2(p, w0, w1);
  ld_ll2(p + 2, w2, w3);
  if (tag_of(w0) != tag || tag_of(w1) != tag || tag_of(w2) != tag || tag_of(w3) != tag) {
    const long long t0 = clock64();
    for (unsigned it = 1;; ++it) {
      ld_ll2(p, w0, w1);
      ld_ll2(p + 2, w2, w3);
      if (tag_of(w0) == tag && tag_of(w1) == tag && tag_of(w2) == tag && tag_of(w3) == tag) break;
      if (clock64() - t0 > budget) { atomicCAS(gerr, 0, kErrWaitTimeoutPeer); return false; }
      if ((it & 255) == 0 && poll_abort(gerr)) return false;
    }
  }
  v[0] = uint32_t(w0); v[1] = uint32_t(w1); v[2] = uint32_t(w2); v[3] = uint32_t(w3);
  return true;
}

// Expert-parallel combine from a GEMM epilogue. A thread holds output feature m of
// a tile row (lanes hold consecutive features) and the value for sorted row `row`;
// lane pairs (m even, m + 1) pack their bf16 values into one tagged word of the
// source rank's combine slot. Call with the whole warp (it shuffles); `active`
// marks lanes whose feature is inside the tile.
struct EpCombDev {
  unsigned long long base[8];
  long long comb_off;
  int cap, kk, H, layers_per_step;
  const int* comb_dst;
  const int64_t* epoch;
  int layer;
};

SP_DEVI uint32_t ep_comb_tag(const EpCombDev& e, int* buf) {
  const u64 x = u64(*e.epoch) * e.layers_per_step + e.layer;
  *buf = int(x & 1);
  return uint32_t(x + 1);
}

SP_DEVI void ep_comb_store(const EpCombDev& e, int buf, uint32_t tag, int row, long long m, float v, bool active) {
  const int dst = __ldg(e.comb_dst + row);
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const uint32_t mine = uint32_t(*reinterpret_cast<const unsigned short*>(&h));
  const uint32_t other = __shfl_down_sync(0xffffffffu, mine, 1);
  if (active && (m & 1) == 0) {
    const int r = dst >> 20, slot = dst & 0xFFFFF;
    u64* w = reinterpret_cast<u64*>(e.base[r] + e.comb_off) + ((long long)buf * e.cap * e.kk + slot) * (e.H / 2) + m / 2;
    st_ll(w, ll_word(mine | (other << 16), tag));
  }
}

}  // namespace sp
