// Peer exchange buffer of a fused row-split linear + all-reduce over NVLink.
//
// Every rank owns one buffer per all-reduce site, laid out identically on all
// ranks and mapped into the other ranks' address spaces (CUDA IPC, plain
// peer mappings):
//   data  [2 parities][world][tokens_max][features] of (fp32 bits, tag) pairs,
//         8 bytes each, written by the ranks' linears
//   sync  [epoch, consumer ticket] uint32, this rank only
// Call e of a site uses parity e & 1 and tag e + 1.  The linear of rank r
// stores each fp32 partial of a (token, feature) together with the tag as one
// 8-byte store into data[parity][r] of every rank: an aligned 8-byte store is
// never torn, so a reader that sees the tag sees that call's value, and no
// fence or separate flag is needed (a system-scope fence after the stores
// cost microseconds per launch).  The consumer on each rank reads
// data[parity][0..world) of its own buffer, waits (bounded) for any word
// whose tag is not yet e + 1, sums in rank order and, with its last CTA,
// advances its epoch.  A rank writes call e + 2 into a parity only after it
// has consumed call e + 1, which needs every rank's call-(e + 1) partial,
// which each rank produces only after it has consumed call e: so no rank
// overwrites words its peers have not read.  The buffer starts zeroed, and
// tag 0 is never a call's.
#pragma once

#include <cstdint>

namespace dsb {

struct PeerLayout {
  int64_t data_bytes, sync_off, total;
  __host__ __device__ PeerLayout(int world, int tokens_max, int features) {
    data_bytes = 2ll * world * tokens_max * features * 8;
    sync_off = (data_bytes + 127) / 128 * 128;
    total = sync_off + 128;
  }
};

constexpr int kPeerMaxWorld = 8;
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // 2 s for the peers' partials of one call

// One (value, tag) word, stored in one 8-byte access visible to the peers.
__device__ __forceinline__ void st_tagged(void *p, float v, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)),
               "r"(tag)
               : "memory");
}

// Eight consecutive (value, tag) words of this rank's buffer into v[0..7],
// once all of them carry `tag`: polled (bounded by time, checked every 64
// polls, with a poll count as a backstop); false when the bound ran out.
// With wait false (a wait of this thread already ran out) one poll only.
__device__ __forceinline__ bool ld_tagged8(const void *p, uint32_t tag, float (&v)[8],
                                           bool wait = true) {
  uint64_t t0 = 0;
  for (int i = 0; i < (wait ? (1 << 24) : 1); ++i) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t a, ta, b, tb;
      asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(a), "=r"(ta), "=r"(b), "=r"(tb)
                   : "l"(static_cast<const uint8_t *>(p) + 16 * k)
                   : "memory");
      v[2 * k] = __uint_as_float(a);
      v[2 * k + 1] = __uint_as_float(b);
      all = all && ta == tag && tb == tag;
    }
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
