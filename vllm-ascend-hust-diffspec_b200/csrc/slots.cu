// Request slots on the device: the canonical-row bookkeeping of the draft
// cache (set_active_requests, diffspec/runtime.py:755-778) as one kernel
// over a device slot table, so a batch change costs one launch and no host
// state beyond the request-id -> key interning.
//
// Semantics kept from the reference:
//  * a request keeps its slot for as long as it stays in the batch, whatever
//    its row (batch reorder moves nothing);
//  * every slot whose request left the batch is released first, and its
//    per-slot state reset (working length 0; selection count -1, i.e. no
//    selection);
//  * requests new to the table then take the lowest free slots, in batch
//    order of their first occurrence (a duplicated id shares its slot);
//  * when the free slots run out, the new requests in batch order that still
//    fit are assigned, the rest are not (the reference raises at the first
//    one that does not fit, after the same releases and assignments).
#include <cstdint>

#include "common.cuh"

namespace dsb {
namespace {

constexpr int kSlotThreads = 1024;
constexpr int kSlotMax = 4096;  // slots of the table and requests of one call

// Exclusive prefix sum of a[0..n) in shared memory (n <= 4 * blockDim.x);
// returns the total.  Every thread of the block calls it.
__device__ int block_exclusive_scan(int32_t *a, int n, int32_t *warp_tot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int base = tid * 4;
  int v[4], s = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = (base + k < n) ? a[base + k] : 0;
    s += v[k];
  }
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < nw) warp_tot[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int run = incl - s + (warp > 0 ? warp_tot[warp - 1] : 0);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (base + k < n) a[base + k] = run;
    run += v[k];
  }
  const int total = warp_tot[(blockDim.x >> 5) - 1];
  __syncthreads();
  return total;
}

// One CTA.  slot_keys[s] is the key of the request owning slot s, or
// negative when the slot is free.  Work is O(n * S / threads) compares,
// which for the sizes of a serving batch is a few microseconds; it runs only
// when the batch changes.
__global__ void __launch_bounds__(kSlotThreads)
assign_slots_kernel(int64_t *__restrict__ slot_keys, int S,
                    const int64_t *__restrict__ request_keys, int n,
                    int32_t *__restrict__ active_slots, int32_t *__restrict__ sel_count,
                    int32_t *__restrict__ working_lens, int32_t *__restrict__ status,
                    int32_t *error_flag) {
  extern __shared__ int64_t slot_smem[];
  int64_t *tkey = slot_smem;                                    // [S] table keys
  int64_t *rkey = tkey + S;                                     // [n] request keys
  int32_t *first = reinterpret_cast<int32_t *>(rkey + n);       // [n] first occurrence
  int32_t *rslot = first + n;                                   // [n] slot of a first occurrence
  int32_t *newrank = rslot + n;                                 // [n] new flag -> rank
  int32_t *isfree = newrank + n;                                // [S] free after the releases
  int32_t *freerank = isfree + S;                               // [S] rank among the free slots
  int32_t *freelist = freerank + S;                             // [S] free slots, ascending
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t bad;
  const int tid = threadIdx.x;

  pdl_begin();
  if (tid == 0) bad = 0;
  for (int s = tid; s < S; s += blockDim.x) tkey[s] = slot_keys[s];
  for (int i = tid; i < n; i += blockDim.x) rkey[i] = request_keys[i];
  __syncthreads();

  // first occurrence of every request key, in batch order
  for (int i = tid; i < n; i += blockDim.x) {
    const int64_t k = rkey[i];
    int f = i;
    for (int j = 0; j < i; ++j)
      if (rkey[j] == k) {
        f = j;
        break;
      }
    first[i] = f;
    if (k < 0) bad = 1;  // negative keys mark free slots: not a request key
  }
  // release every slot whose request left the batch
  for (int s = tid; s < S; s += blockDim.x) {
    const int64_t k = tkey[s];
    int is_free = k < 0;
    if (!is_free) {
      bool kept = false;
      for (int i = 0; i < n && !kept; ++i) kept = rkey[i] == k;
      if (!kept) {
        if (sel_count != nullptr) sel_count[s] = -1;
        if (working_lens != nullptr) working_lens[s] = 0;
        is_free = 1;
      }
    }
    isfree[s] = is_free;
    freerank[s] = is_free;
  }
  __syncthreads();
  // slot already held by each first occurrence (a kept slot: its key is in
  // the batch), else a new request
  for (int i = tid; i < n; i += blockDim.x) {
    int slot = -1, is_new = 0;
    if (first[i] == i && rkey[i] >= 0) {
      for (int s = 0; s < S; ++s)
        if (tkey[s] == rkey[i]) {
          slot = s;
          break;
        }
      is_new = slot < 0;
    }
    rslot[i] = slot;
    newrank[i] = is_new;
  }
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x)  // released keys leave the table
    if (isfree[s]) tkey[s] = -1;
  const int nfree = block_exclusive_scan(freerank, S, warp_tot);
  for (int s = tid; s < S; s += blockDim.x)
    if (isfree[s]) freelist[freerank[s]] = s;  // ascending: rank order is slot order
  __syncthreads();
  // rslot[i] doubles as the new-flag store during the scan of newrank
  for (int i = tid; i < n; i += blockDim.x)
    if (rslot[i] < 0 && first[i] == i && rkey[i] >= 0) rslot[i] = -2;  // new
  __syncthreads();
  const int nnew = block_exclusive_scan(newrank, n, warp_tot);
  // only freelist[0, nfree) is read, and every rank below nfree belongs to
  // exactly one free slot
  for (int i = tid; i < n; i += blockDim.x) {
    if (rslot[i] != -2) continue;
    const int r = newrank[i];
    if (r < nfree) {
      const int s = freelist[r];
      rslot[i] = s;
      tkey[s] = rkey[i];
    } else {
      rslot[i] = -1;  // slots exhausted
    }
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) active_slots[i] = rslot[first[i]];
  for (int s = tid; s < S; s += blockDim.x) slot_keys[s] = tkey[s];
  if (tid == 0) {
    if (status != nullptr) {
      status[0] = nnew > nfree ? nnew - nfree : 0;  // new requests left without a slot
      status[1] = nfree - min(nnew, nfree);         // free slots after the call
    }
    if (bad) flag_error(error_flag, DSB_FLAG_SLOT);
  }
}

__global__ void rows_to_slots_kernel(const int32_t *__restrict__ active_slots, int num_active,
                                     const int32_t *__restrict__ rows, int n,
                                     int32_t *__restrict__ slots, int32_t *error_flag) {
  pdl_begin();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rows[i];
  if (r < 0 || r >= num_active) {
    slots[i] = -1;  // no cache row
    flag_error(error_flag, DSB_FLAG_SLOT);
    return;
  }
  slots[i] = active_slots[r];
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_assign_request_slots(int64_t *slot_keys, int32_t num_slots,
                                        const int64_t *request_keys, int32_t num_requests,
                                        int32_t *active_slots, int32_t *sel_count,
                                        int32_t *working_lens, int32_t *status,
                                        int32_t *error_flag, void *stream) {
  if (num_slots <= 0 || num_slots > kSlotMax || num_requests < 0 || num_requests > kSlotMax)
    return fail(DSB_ERR_INVALID, "num_slots must be in [1, 4096] and num_requests in [0, 4096]");
  if (!slot_keys || (num_requests > 0 && (!request_keys || !active_slots)))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  const size_t smem = (size_t)(num_slots + num_requests) * 8 +
                      (size_t)(3 * num_requests + 3 * num_slots) * 4;
  const void *kern = (const void *)assign_slots_kernel;
  if (ensure_smem(kern, smem) != DSB_OK) return DSB_ERR_CUDA;
  launch_kernel(assign_slots_kernel, dim3(1), dim3(kSlotThreads), smem, as_stream(stream),
                slot_keys, (int)num_slots, request_keys, (int)num_requests, active_slots,
                sel_count, working_lens, status, error_flag);
  return check_launch("assign_slots_kernel");
}

extern "C" int dsb_rows_to_slots(const int32_t *active_slots, int32_t num_active,
                                 const int32_t *rows, int32_t n, int32_t *slots,
                                 int32_t *error_flag, void *stream) {
  if (n < 0 || num_active < 0) return fail(DSB_ERR_INVALID, "negative count");
  if (n == 0) return DSB_OK;
  if (!active_slots || !rows || !slots) return fail(DSB_ERR_INVALID, "null pointer argument");
  launch_kernel(rows_to_slots_kernel, dim3((n + 255) / 256), dim3(256), 0, as_stream(stream),
                active_slots, (int)num_active, rows, (int)n, slots, error_flag);
  return check_launch("rows_to_slots_kernel");
}
