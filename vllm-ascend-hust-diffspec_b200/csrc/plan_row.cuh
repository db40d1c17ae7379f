// History-plan row of one request, shared by the plan kernel and the fused
// plan + rebuild launch: _history_plan_host, diffspec/runtime.py:1713-1735.
//
// History ends just before the root (history_end = committed_len - 1).  The
// rolling tail is the last min(window, history_budget) history tokens (window
// = one chunk in the reference; a longer rolling recent window is the window
// mode, which has no reference counterpart); the
// selected chunks (ascending, the newest last) contribute their tokens that
// lie before both the tail and the newest selected chunk's start, keeping the
// last history_budget - tail of them (prefix_drop counts the dropped oldest
// ones).  A slot without any retrieval yet (count < 0) takes the most recent
// history_budget tokens.
#pragma once

#include "common.cuh"

namespace dsb {

struct PlanRow {
  int64_t hlen, tail_start, prefix_len, prefix_drop;
  int n_chunks;  // selected chunk ids the row carries (capped by the plan width)
};

// One warp computes the row: lanes read the slot's selected chunks in
// parallel and a warp reduction forms the prefix length.  All 32 lanes call
// it with the same arguments and get the same result.  `ch` is the slot's
// row of selected chunk ids, `cnt` its count.
__device__ __forceinline__ PlanRow plan_row_warp(int committed_len, int cnt, const int32_t *ch,
                                                 int sel_stride, int C, int HB, int window,
                                                 int plan_width, int lane, int32_t *err) {
  PlanRow pr;
  const int64_t he = max(0, committed_len - 1);  // history ends before the root
  const int n_sel = min(max(cnt, 0), sel_stride);
  pr.n_chunks = n_sel;
  if (5 + pr.n_chunks > plan_width) {
    if (lane == 0) flag_error(err, DSB_FLAG_CAPACITY);
    pr.n_chunks = plan_width - 5;
  }
  const int64_t tail_len = min(he, (int64_t)min(window, HB));
  pr.prefix_len = 0;
  pr.prefix_drop = 0;
  if (cnt < 0) {  // no retrieval yet: the most recent history_budget tokens
    pr.hlen = min(he, (int64_t)HB);
    pr.tail_start = he - pr.hlen;
  } else if (cnt == 0) {
    pr.hlen = tail_len;
    pr.tail_start = he - tail_len;
  } else {
    pr.tail_start = he - tail_len;
    const int64_t prefix_end = min(pr.tail_start, (int64_t)ch[n_sel - 1] * C);
    int64_t part = 0;
    for (int i = lane; i < n_sel; i += 32)
      part += max((int64_t)0, min((int64_t)C, prefix_end - (int64_t)ch[i] * C));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    pr.prefix_len = min(part, (int64_t)HB - tail_len);
    pr.prefix_drop = part - pr.prefix_len;
    pr.hlen = pr.prefix_len + tail_len;
  }
  return pr;
}

// Plan row value i: [slot, history_len, tail_start, prefix_len, prefix_drop,
// chunk ids..., zeros].
__device__ __forceinline__ int64_t plan_row_value(const PlanRow &pr, int slot, const int32_t *ch,
                                                  int i) {
  if (i == 0) return slot;
  if (i == 1) return pr.hlen;
  if (i == 2) return pr.tail_start;
  if (i == 3) return pr.prefix_len;
  if (i == 4) return pr.prefix_drop;
  return (i - 5 < pr.n_chunks) ? ch[i - 5] : 0;
}

}  // namespace dsb
