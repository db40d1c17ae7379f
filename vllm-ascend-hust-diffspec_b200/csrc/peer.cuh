// Peer exchange buffer of a fused row-split linear + all-reduce over NVLink.
//
// Every rank owns one buffer per all-reduce site, laid out identically on all
// ranks and mapped into the other ranks' address spaces (CUDA IPC, plain
// peer mappings):
//   data  [2 parities][world][tokens_max][features] fp32  written by the ranks' linears
//   flags [2 parities][world] uint32                      written by the ranks' linears
//   sync  [epoch, producer ticket, consumer ticket] uint32 this rank only
// Call e of a site uses parity e & 1.  The linear of rank r stores its fp32
// partial of every (token, feature) into data[parity][r] of every rank, and
// the last of its CTAs to finish sets flags[parity][r] = e + 1 on every rank
// (release at system scope).  The consumer on each rank waits (bounded) until
// all of its flags[parity][*] equal e + 1, sums data[parity][0..world) in
// rank order and, with its last CTA, advances its epoch.  A rank writes call
// e + 2 into a parity only after it has consumed call e + 1, which needs
// every rank's call-(e + 1) partial, which each rank produces only after it
// has consumed call e: so no rank overwrites data its peers have not read.
#pragma once

#include <cstdint>

namespace dsb {

struct PeerLayout {
  int64_t data_bytes, flags_off, sync_off, total;
  __host__ __device__ PeerLayout(int world, int tokens_max, int features) {
    data_bytes = 2ll * world * tokens_max * features * 4;
    flags_off = (data_bytes + 127) / 128 * 128;
    sync_off = flags_off + (2ll * world * 4 + 127) / 128 * 128;
    total = sync_off + 128;
  }
};

constexpr int kPeerMaxWorld = 8;
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // 2 s for the peers' partials of one call

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (wall clock, checked every 64 polls, with a poll count as a
// backstop) until flags[0..world) all equal `want`; false when the bound ran
// out.
__device__ __forceinline__ bool peer_wait_flags(const uint32_t *flags, int world, uint32_t want) {
  uint64_t t0 = 0;
  for (int i = 0; i < (1 << 24); ++i) {
    bool all = true;
    for (int q = 0; q < world && all; ++q) all = ld_acquire_sys(flags + q) == want;
    if (all) return true;
    if ((i & 63) == 0) {
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (i == 0) t0 = now;
      else if (now - t0 > kPeerWaitNs) return false;
    }
  }
  return false;
}

}  // namespace dsb
