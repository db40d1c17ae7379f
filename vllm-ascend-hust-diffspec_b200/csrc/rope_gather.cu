// Fused gather + local-position RoPE + write (DiffSpec rows A6 and A7).
//
// Reference: _rebuild_compact_kv_kernel / rebuild_compact_kv_from_plan,
// diffspec/compact_kv.py:8-242 (grid (rows, heads, cdiv(width, 16)), one head
// and 16 tokens per program, cos/sin re-read per head) and
// gather_raw_kv_with_local_rope, diffspec/kernels.py:153-210 (index_select
// followed by a separate in-place RoPE pass).
//
// B200 design: a warp owns U whole token rows (all kv heads, K and V).  The
// raw rows are contiguous [heads * head_dim] runs, so each lane issues 16-byte
// cp.async copies into a per-warp shared-memory stage (perfectly coalesced,
// no register staging, U * 2 rows in flight per warp).  The warp then writes
// V straight back out and K rotated at the local position, reading the RoPE
// partner element from the staged row, so one HBM read and one HBM write per
// byte is all the kernel moves.  RoPE math is fp32 with both products rounded
// before the add, i.e. exactly "first * cos - second * sin" evaluated without
// fused multiply-add, then rounded once to the cache dtype.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "plan_row.cuh"

namespace dsb {
namespace {

constexpr int kWarpsRope = 8;

struct RopeArgs {
  const void *src_k, *src_v;
  void *dst_k, *dst_v;
  // rebuild (plan-driven)
  const int64_t *plan;
  int plan_width, num_slots;
  int64_t max_model_len;
  int working_budget, chunk, max_width;
  // gather (paged, index-driven)
  const int32_t *bt;
  int64_t bt_stride, bt_cols, num_blocks;
  int block_size;
  const int64_t *sel;
  int working_tokens;
  // common
  const void *cos_sin;
  int64_t cs_stride, cs_rows;
  int heads, head_dim, rotary_dim, neox, tokens_per_warp;
  int pt_shift;  // bulk kernel: log2 of the positions per CTA
  int vec_rope;  // NeoX with 16-byte-aligned halves and cos/sin rows: vector path
  int cs_bulk;   // bulk kernel: the CTA's cos/sin rows are staged with its K/V rows
  // rebuild from the selection state: the launch computes each row's plan
  // (plan_row_warp) instead of reading it, and CTA 0 of the row writes it out
  int from_sel;
  const int32_t *row_slots, *committed_lens, *sel_chunks, *sel_count;
  int sel_stride, history_budget, window;
  int64_t *plan_out;
  int32_t *hist_out, *wlen_out;
  int chunk_shift, block_shift;  // log2 of chunk / block_size when powers of two, else -1
  int32_t *err;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

template <typename CS>
__device__ __forceinline__ float cs_load(const CS *p) {
  return Elem<CS>::to_f(*p);
}

// N consecutive table entries as floats (aligned vector loads; N * sizeof(CS)
// is 8, 16 or 32 bytes).
// SHARED: p points into shared memory (plain loads instead of the read-only
// global path).
template <typename CS, int N, bool SHARED = false>
__device__ __forceinline__ void cs_load_vec(const CS *p, float (&out)[N]) {
  constexpr int bytes = N * (int)sizeof(CS);
  union {
    uint4 q[bytes >= 16 ? bytes / 16 : 1];
    uint2 d;
    CS e[N];
  } u;
  if constexpr (bytes >= 16) {
#pragma unroll
    for (int i = 0; i < bytes / 16; ++i)
      u.q[i] = SHARED ? reinterpret_cast<const uint4 *>(p)[i] : __ldg(reinterpret_cast<const uint4 *>(p) + i);
  } else {
    u.d = SHARED ? *reinterpret_cast<const uint2 *>(p) : __ldg(reinterpret_cast<const uint2 *>(p));
  }
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = Elem<CS>::to_f(u.e[i]);
}


// Two 16-bit elements of a 32-bit word as floats, and back with one
// round-to-nearest-even conversion per pair.
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <> struct Pair<__half> {
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

// out = x * c + y * s_signed, element-wise over 8 packed 16-bit values; the
// caller passes s_signed = -sin for the first rotary half, so this equals
// x*cos - y*sin there and x*cos + y*sin in the second half (products rounded
// before the add, as in the unfused reference arithmetic).
template <typename T>
__device__ __forceinline__ uint4 rotate8(const uint4 &x, const uint4 &y, const float (&c)[8],
                                         const float (&s)[8]) {
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
  uint32_t o[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float2 xf = Pair<T>::unpack(xs[w]), yf = Pair<T>::unpack(ys[w]);
    const float r0 = __fmul_rn(xf.x, c[2 * w]) + __fmul_rn(yf.x, s[2 * w]);
    const float r1 = __fmul_rn(xf.y, c[2 * w + 1]) + __fmul_rn(yf.y, s[2 * w + 1]);
    o[w] = Pair<T>::pack(r0, r1);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <typename T, typename CS, bool GATHER, int DH>
__global__ void __launch_bounds__(kWarpsRope * 32, 3) rope_rows_kernel(const RopeArgs a) {
  pdl_begin();
  // DH: head_dim known at compile time (64, 128, 256), or 0 for any other.
  const int head_dim = DH ? DH : a.head_dim;
  extern __shared__ uint4 stage[];
  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = a.tokens_per_warp;
  const int row_elems = a.heads * head_dim;
  const int row_vecs = row_elems / VE;
  uint4 *wstage = stage + (size_t)warp * 2 * U * 2 * row_vecs;  // two batches per warp
  const T *src_k = static_cast<const T *>(a.src_k);
  const T *src_v = static_cast<const T *>(a.src_v);
  T *dst_k = static_cast<T *>(a.dst_k);
  T *dst_v = static_cast<T *>(a.dst_v);
  const CS *cs = static_cast<const CS *>(a.cos_sin);
  const int r = blockIdx.y;

  // Row descriptor.
  int64_t slot = 0, hlen = 0, tail_start = 0, prefix_len = 0, drop = 0;
  const int64_t *chunks = nullptr;
  int n_plan_chunks = 0;
  if (!GATHER) {
    const int64_t *pr = a.plan + (int64_t)r * a.plan_width;
    slot = pr[0];
    hlen = pr[1];
    tail_start = pr[2];
    prefix_len = pr[3];
    drop = pr[4];
    chunks = pr + 5;
    n_plan_chunks = a.plan_width - 5;
    const int64_t cap = min((int64_t)a.max_width, (int64_t)a.working_budget);
    if (slot < 0 || slot >= a.num_slots || hlen < 0 || prefix_len < 0 || prefix_len > hlen ||
        drop < 0 || hlen > cap) {
      if (lane == 0 && warp == 0 && blockIdx.x == 0)
        flag_error(a.err, (slot < 0 || slot >= a.num_slots) ? DSB_FLAG_SLOT : DSB_FLAG_PLAN);
      if (slot < 0 || slot >= a.num_slots) return;
      hlen = max((int64_t)0, min(hlen, cap));
      prefix_len = max((int64_t)0, min(prefix_len, hlen));
      drop = max((int64_t)0, drop);
    }
  }
  const int64_t width = GATHER ? a.working_tokens : hlen;

  // Source rows of local position p: 1 = copy, 2 = zero row (gather
  // padding), 0 = skip (bad plan data, flagged).
  auto source = [&](int64_t p, const T *&rk, const T *&rv) -> int {
    if (!GATHER) {
      int64_t abs_pos;
      bool ok = true;
      if (p < prefix_len) {
        const int q = (int)(p + drop);
        const int ci = a.chunk_shift >= 0 ? q >> a.chunk_shift : q / a.chunk;
        if (ci >= n_plan_chunks) ok = false;
        abs_pos = ok ? chunks[ci] * a.chunk + (q - ci * a.chunk) : 0;
      } else {
        abs_pos = tail_start + p - prefix_len;
      }
      if (!ok || abs_pos < 0 || abs_pos >= a.max_model_len) {
        if (lane == 0) flag_error(a.err, ok ? DSB_FLAG_POSITION : DSB_FLAG_PLAN);
        return 0;
      }
      const int64_t off = (slot * a.max_model_len + abs_pos) * row_elems;
      rk = src_k + off;
      rv = src_v + off;
      return 1;
    }
    const int64_t idx = a.sel[(int64_t)r * a.working_tokens + p];
    if (idx < 0) return 2;
    int64_t lb, in_block;
    if (a.block_shift >= 0) {
      lb = idx >> a.block_shift;
      in_block = idx & ((1LL << a.block_shift) - 1);
    } else {
      lb = idx / a.block_size;
      in_block = idx - lb * a.block_size;
    }
    const int64_t pb = (lb < a.bt_cols) ? a.bt[(int64_t)r * a.bt_stride + lb] : -1;
    if (pb < 0 || pb >= a.num_blocks) {
      if (lane == 0) flag_error(a.err, DSB_FLAG_BLOCK);
      return 2;
    }
    const int64_t off = (pb * a.block_size + in_block) * row_elems;
    rk = src_k + off;
    rv = src_v + off;
    return 1;
  };
  // Stage the U rows (K then V) of one batch with 16-byte cp.async.
  auto stage_batch = [&](int64_t pb, uint4 *buf) {
    for (int j = 0; j < U; ++j) {
      const int64_t p = pb + j;
      if (p >= width) break;
      const T *rk = nullptr, *rv = nullptr;
      const int kind = source(p, rk, rv);
      if (kind == 0) continue;
      uint4 *sk = buf + (size_t)j * 2 * row_vecs;
      uint4 *sv = sk + row_vecs;
      for (int v = lane; v < row_vecs; v += 32) {
        if (kind == 2) {
          sk[v] = make_uint4(0, 0, 0, 0);
          sv[v] = make_uint4(0, 0, 0, 0);
        } else {
          cp_async16(sk + v, reinterpret_cast<const uint4 *>(rk) + v);
          cp_async16(sv + v, reinterpret_cast<const uint4 *>(rv) + v);
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int rot = a.rotary_dim, half = rot / 2;
  // Write V as is and K rotated at local position p.
  auto write_batch = [&](int64_t pb, const uint4 *buf) {
    for (int j = 0; j < U; ++j) {
      const int64_t p = pb + j;
      if (p >= width) break;
      if (!GATHER) {  // skip rows whose source was rejected when staging
        bool ok = true;
        int64_t abs_pos;
        if (p < prefix_len) {
          const int q = (int)(p + drop);
          const int ci = a.chunk_shift >= 0 ? q >> a.chunk_shift : q / a.chunk;
          ok = ci < n_plan_chunks;
          abs_pos = ok ? chunks[ci] * a.chunk + (q - ci * a.chunk) : 0;
        } else {
          abs_pos = tail_start + p - prefix_len;
        }
        if (!ok || abs_pos < 0 || abs_pos >= a.max_model_len) continue;
      }
      const uint4 *sk = buf + (size_t)j * 2 * row_vecs;
      const uint4 *sv = sk + row_vecs;
      const T *kx = reinterpret_cast<const T *>(sk);
      const CS *csr = cs + p * a.cs_stride;
      // With a compile-time head_dim whose vectors-per-head divide 32, every
      // vector of this lane sits at the same head offset: one cos/sin load.
      constexpr int kHeadVecs = DH ? DH / VE : 1;
      constexpr bool kSameOffset = DH != 0 && (32 % kHeadVecs) == 0;
      float cvec[VE], svec[VE];  // svec holds -sin in the first rotary half
      if (kSameOffset && a.vec_rope) {
        const int d0 = (lane % kHeadVecs) * VE;
        if (d0 < rot) {
          const int i0 = d0 < half ? d0 : d0 - half;
          cs_load_vec<CS, VE>(csr + i0, cvec);
          cs_load_vec<CS, VE>(csr + half + i0, svec);
          if (d0 < half) {
#pragma unroll
            for (int e = 0; e < VE; ++e) svec[e] = -svec[e];
          }
        }
      }
      const int64_t dst_tok = GATHER ? ((int64_t)r * a.working_tokens + p) * row_elems
                                     : (slot * a.heads * (int64_t)a.working_budget + p) * head_dim;
      for (int v = lane; v < row_vecs; v += 32) {
        const int e0 = v * VE;
        const int h = e0 / head_dim, d0 = e0 - h * head_dim;
        const int64_t dst_off =
            GATHER ? dst_tok + e0 : dst_tok + (int64_t)h * a.working_budget * head_dim + d0;
        stg_stream(dst_v + dst_off, sv[v]);
        if (d0 >= rot) {
          stg_stream(dst_k + dst_off, sk[v]);
          continue;
        }
        const T *hx = kx + h * head_dim;
        union {
          uint4 u;
          T e[VE];
        } out;
        out.u = sk[v];
        if constexpr (kSameOffset && sizeof(T) == 2) {
          if (a.vec_rope) {  // packed path with the per-token cos / signed sin
            const bool first = d0 < half;
            const uint4 par = sk[first ? v + half / VE : v - half / VE];
            stg_stream(dst_k + dst_off, rotate8<T>(out.u, par, cvec, svec));
            continue;
          }
        }
        if (a.vec_rope) {  // whole vector rotary; partner is the vector half away
          const bool first = d0 < half;
          const int i0 = first ? d0 : d0 - half;
          union {
            uint4 u;
            T e[VE];
          } par;
          par.u = sk[first ? v + half / VE : v - half / VE];
          float c[VE], sn[VE];
          cs_load_vec<CS, VE>(csr + i0, c);
          cs_load_vec<CS, VE>(csr + half + i0, sn);
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float x = Elem<T>::to_f(out.e[e]), y = Elem<T>::to_f(par.e[e]);
            const float rr = first ? __fmul_rn(x, c[e]) - __fmul_rn(y, sn[e])
                                   : __fmul_rn(x, c[e]) + __fmul_rn(y, sn[e]);
            out.e[e] = Elem<T>::from_f(rr);
          }
          stg_stream(dst_k + dst_off, out.u);
          continue;
        }
#pragma unroll
        for (int e = 0; e < VE; ++e) {
          const int d = d0 + e;
          if (d >= rot) break;
          int i;
          float x1, x2;
          bool first;
          if (a.neox) {
            first = d < half;
            i = first ? d : d - half;
            x1 = Elem<T>::to_f(hx[i]);
            x2 = Elem<T>::to_f(hx[i + half]);
          } else {
            first = (d & 1) == 0;
            i = d >> 1;
            x1 = Elem<T>::to_f(hx[2 * i]);
            x2 = Elem<T>::to_f(hx[2 * i + 1]);
          }
          const float c = cs_load(csr + i), sn = cs_load(csr + half + i);
          const float y = first ? __fmul_rn(x1, c) - __fmul_rn(x2, sn)
                                : __fmul_rn(x2, c) + __fmul_rn(x1, sn);
          out.e[e] = Elem<T>::from_f(y);
        }
        stg_stream(dst_k + dst_off, out.u);
      }
    }
  };

  // Grid-stride over batches of U positions, double-buffered: batch b + 1 is
  // copied while batch b is rotated and written.
  auto batch_start = [&](int b) {
    return ((int64_t)b * gridDim.x + blockIdx.x) * kWarpsRope * U + (int64_t)warp * U;
  };
  uint4 *bufs[2] = {wstage, wstage + (size_t)U * 2 * row_vecs};
  if (batch_start(0) < width) {
    stage_batch(batch_start(0), bufs[0]);
    for (int b = 0; batch_start(b) < width; ++b) {
      const bool more = batch_start(b + 1) < width;
      if (more) stage_batch(batch_start(b + 1), bufs[(b + 1) & 1]);
      if (more) asm volatile("cp.async.wait_group 1;" ::: "memory");
      else asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      write_batch(batch_start(b), bufs[b & 1]);
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy variant (the default for 16-bit caches with head_dim 64/128/256).
// One CTA owns PT = 1 << pt_shift (<= 64) consecutive local positions of one
// row.  Warp 0 decodes the source of each position once (lane t: positions t
// and t + 32) and issues 1-D bulk copies (TMA) of the K rows and V rows (all
// kv heads) into shared memory, one copy per run of consecutive source rows
// (a selected chunk or the rolling tail is one run), all completing on one
// mbarrier.  The block then writes V out unchanged and K rotated: for NeoX
// with 16-byte halves a thread owns one (position, 8-element pair of vectors)
// item, loads its cos/sin vectors once and reuses them for every kv head.
constexpr int kBulkThreads = 256;

// Shared-memory layout of the bulk kernel: kBulkStages stages of [K rows, V
// rows (PT each), PT int32 kinds, the cos/sin rows], then the stages'
// mbarriers and the row's int64 chunk ids.
#ifndef DSB_BULK_STAGES
#define DSB_BULK_STAGES 2
#endif
constexpr int kBulkStages = DSB_BULK_STAGES;
struct BulkLayout {
  size_t v, kind, cs, stage;  // offsets inside a stage, and its size
  size_t bars, chunks, total;
};
__host__ __device__ inline BulkLayout bulk_smem_layout(int pt, int64_t row_bytes, int n_chunks,
                                                       int64_t cs_bytes) {
  BulkLayout l;
  l.v = (size_t)pt * (size_t)row_bytes;  // row_bytes is a multiple of 16
  l.kind = 2 * (size_t)pt * (size_t)row_bytes;
  l.cs = (l.kind + 4 * (size_t)pt + 15) & ~(size_t)15;
  l.stage = (l.cs + (size_t)cs_bytes + 15) & ~(size_t)15;
  l.bars = kBulkStages * l.stage;
  l.chunks = l.bars + 8 * kBulkStages;
  l.total = l.chunks + 8 * (size_t)(n_chunks > 0 ? n_chunks : 0);
  return l;
}

// Bulk-copy rebuild / gather (the default for 16-bit caches with head_dim
// 64/128/256).  A CTA owns one row and the position blocks b = blockIdx.x,
// blockIdx.x + gridDim.x, ... of it (PT = 1 << pt_shift <= 64 positions
// each), streamed through two stages: while the block in one stage is
// rotated and written, the next block's rows are already in flight into the
// other.  Warp 0 decodes the sources of a block (lane t: positions t and
// t + 32) and issues 1-D bulk copies (TMA) of the K rows and V rows (all kv
// heads), one per run of consecutive source rows (a selected chunk or the
// rolling tail is one run), plus one copy of the block's cos/sin rows, all
// completing on the stage's mbarrier.  The block then writes V out unchanged
// and K rotated: for NeoX with 16-byte halves one thread per (head, token,
// 8-element pair of vectors) item.  The row descriptor (plan row, read or
// computed from the selection state) is decoded once per CTA.
template <typename T, typename CS, bool GATHER, int DH>
__global__ void __launch_bounds__(kBulkThreads) rope_bulk_kernel(const RopeArgs a) {
  static_assert(sizeof(T) == 2 && DH > 0, "16-bit caches with a compile-time head_dim");
  constexpr int VE = 8;           // elements per 16-byte vector
  constexpr int DV = DH / VE;     // vectors per head row
  extern __shared__ __align__(16) uint8_t bulk_smem[];
  const int tid = threadIdx.x, lane = tid & 31;
  const int PT = 1 << a.pt_shift;
  const int heads = a.heads;
  const int row_elems = heads * DH;
  const uint32_t row_bytes = (uint32_t)row_elems * 2u;
  const int64_t cs_row_bytes = a.cs_stride * (int64_t)sizeof(CS);
  const BulkLayout lay = bulk_smem_layout(PT, row_bytes, GATHER ? 0 : a.plan_width - 5,
                                          a.cs_bulk ? PT * cs_row_bytes : 0);
  int64_t *s_chunks = reinterpret_cast<int64_t *>(bulk_smem + lay.chunks);
  const uint32_t bar0 = smem_u32(bulk_smem + lay.bars);
  __shared__ int64_t s_desc[5];
  const int r = blockIdx.y;
  if (tid == 0) {  // no global data: overlaps the previous kernel
    for (int s = 0; s < kBulkStages; ++s) mbar_init(bar0 + 8 * s);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_begin();
  // Row descriptor (rebuild: plan row, read or computed here; gather: the
  // row's index vector).  Warp 0 stages it and the row's chunk ids in shared
  // memory.
  int64_t slot = 0, hlen = 0, tail_start = 0, prefix_len = 0, drop = 0;
  const int64_t *chunks = s_chunks;
  const int n_plan_chunks = GATHER ? 0 : a.plan_width - 5;
  if (!GATHER) {
    if (tid < 32) {
      if (a.from_sel) {
        const int sl = (a.row_slots != nullptr) ? a.row_slots[r] : r;
        if (sl < 0 || sl >= a.num_slots) {
          if (blockIdx.x == 0) {
            if (lane == 0) flag_error(a.err, DSB_FLAG_SLOT);
            if (a.plan_out != nullptr)
              for (int i = lane; i < a.plan_width; i += 32) a.plan_out[(int64_t)r * a.plan_width + i] = 0;
            if (lane == 0 && a.hist_out != nullptr) a.hist_out[r] = 0;
          }
          if (lane == 0) {  // nothing to rebuild for this row
            s_desc[0] = 0;
            s_desc[1] = 0;
            s_desc[2] = 0;
            s_desc[3] = 0;
            s_desc[4] = 0;
          }
        } else {
          const int32_t *ch = a.sel_chunks + (int64_t)sl * a.sel_stride;
          const PlanRow pr = plan_row_warp(a.committed_lens[r], a.sel_count[sl], ch, a.sel_stride,
                                           a.chunk, a.history_budget, a.window, a.plan_width, lane,
                                           blockIdx.x == 0 ? a.err : nullptr);
          for (int i = lane; i < n_plan_chunks; i += 32) s_chunks[i] = plan_row_value(pr, sl, ch, 5 + i);
          if (blockIdx.x == 0) {
            if (a.plan_out != nullptr)
              for (int i = lane; i < a.plan_width; i += 32)
                a.plan_out[(int64_t)r * a.plan_width + i] = plan_row_value(pr, sl, ch, i);
            if (lane == 0 && a.hist_out != nullptr) a.hist_out[r] = (int32_t)pr.hlen;
            if (lane == 0 && a.wlen_out != nullptr) a.wlen_out[sl] = (int32_t)pr.hlen;
          }
          if (lane == 0) {
            s_desc[0] = sl;
            s_desc[1] = pr.hlen;
            s_desc[2] = pr.tail_start;
            s_desc[3] = pr.prefix_len;
            s_desc[4] = pr.prefix_drop;
          }
        }
      } else {
        const int64_t *pr = a.plan + (int64_t)r * a.plan_width;
        if (lane < 5) s_desc[lane] = pr[lane];
        for (int i = lane; i < n_plan_chunks; i += 32) s_chunks[i] = pr[5 + i];
      }
    }
    __syncthreads();
    slot = s_desc[0];
    hlen = s_desc[1];
    tail_start = s_desc[2];
    prefix_len = s_desc[3];
    drop = s_desc[4];
    const int64_t cap = min((int64_t)a.max_width, (int64_t)a.working_budget);
    if (slot < 0 || slot >= a.num_slots || hlen < 0 || prefix_len < 0 || prefix_len > hlen ||
        drop < 0 || hlen > cap) {
      if (tid == 0 && blockIdx.x == 0)
        flag_error(a.err, (slot < 0 || slot >= a.num_slots) ? DSB_FLAG_SLOT : DSB_FLAG_PLAN);
      if (slot < 0 || slot >= a.num_slots) return;
      hlen = max((int64_t)0, min(hlen, cap));
      prefix_len = max((int64_t)0, min(prefix_len, hlen));
      drop = max((int64_t)0, drop);
    }
  }
  if (GATHER) __syncthreads();  // the mbarrier initialisation is visible
  const int64_t width = GATHER ? a.working_tokens : hlen;
  const int nblk = (int)((width + PT - 1) >> a.pt_shift);
  const int n_mine = (int)blockIdx.x < nblk ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  if (n_mine == 0) return;  // CTA-uniform

  // Warp 0: decode block i of this CTA and start its copies into stage i % 2.
  auto issue = [&](int i) {
    const int s = i % kBulkStages;
    uint8_t *st = bulk_smem + s * lay.stage;
    uint8_t *sk = st, *sv = st + lay.v;
    int *s_kind = reinterpret_cast<int *>(st + lay.kind);
    const uint32_t bar = bar0 + 8 * s;
    const int64_t p0 = (int64_t)((int)blockIdx.x + i * (int)gridDim.x) << a.pt_shift;
    const int n_tok = (int)min((int64_t)PT, width - p0);
    // Source row of local position p0 + t; kind: 1 = copy the row, 2 = zero
    // row (gather padding / bad block), 0 = skip.
    auto resolve = [&](int t, int64_t &off) -> int {
      if (t >= n_tok) return 0;
      const int64_t p = p0 + t;
      if (!GATHER) {
        int64_t abs_pos = 0;
        bool ok = true;
        if (p < prefix_len) {
          const int q = (int)(p + drop);
          const int ci = a.chunk_shift >= 0 ? q >> a.chunk_shift : q / a.chunk;
          ok = ci < n_plan_chunks;
          if (ok) abs_pos = chunks[ci] * a.chunk + (q - ci * a.chunk);
        } else {
          abs_pos = tail_start + p - prefix_len;
        }
        if (!ok || abs_pos < 0 || abs_pos >= a.max_model_len) {
          flag_error(a.err, ok ? DSB_FLAG_POSITION : DSB_FLAG_PLAN);
          return 0;
        }
        off = (slot * a.max_model_len + abs_pos) * row_elems;
        return 1;
      }
      const int64_t idx = a.sel[(int64_t)r * a.working_tokens + p];
      if (idx < 0) return 2;
      int64_t lb, in_block;
      if (a.block_shift >= 0) {
        lb = idx >> a.block_shift;
        in_block = idx & ((1LL << a.block_shift) - 1);
      } else {
        lb = idx / a.block_size;
        in_block = idx - lb * a.block_size;
      }
      const int64_t pb = (lb < a.bt_cols) ? a.bt[(int64_t)r * a.bt_stride + lb] : -1;
      if (pb < 0 || pb >= a.num_blocks) {
        flag_error(a.err, DSB_FLAG_BLOCK);
        return 2;
      }
      off = (pb * a.block_size + in_block) * row_elems;
      return 1;
    };
    // Tokens lane, lane + 32: consecutive source rows form runs, and each run
    // is one bulk copy of K and one of V (the rows of a run are contiguous
    // in the raw cache and in the stage).
    int kinds[2];
    int64_t offs[2] = {0, 0};
    uint32_t n_loads = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      kinds[j] = (32 * j < PT) ? resolve(lane + 32 * j, offs[j]) : 0;
      n_loads += __popc(__ballot_sync(0xffffffffu, kinds[j] == 1));
    }
    // cos/sin rows of positions p0 .. p0 + n_tok - 1: one contiguous copy
    const uint32_t cs_bytes = a.cs_bulk ? (uint32_t)(n_tok * cs_row_bytes) : 0u;
    if (lane == 0) {
      mbar_expect_tx(bar, n_loads * 2u * row_bytes + cs_bytes);
      if (cs_bytes)
        bulk_load(smem_u32(st + lay.cs), static_cast<const CS *>(a.cos_sin) + p0 * a.cs_stride,
                  cs_bytes, bar);
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = lane + 32 * j;
      const int prev_kind = __shfl_up_sync(0xffffffffu, kinds[j], 1);
      const int64_t prev_off = __shfl_up_sync(0xffffffffu, offs[j], 1);
      const bool cont = lane > 0 && kinds[j] == 1 && prev_kind == 1 && offs[j] == prev_off + row_elems;
      const uint32_t breaks = __ballot_sync(0xffffffffu, !cont);
      if (kinds[j] == 1 && !cont) {
        const uint32_t later = breaks & ~((2u << lane) - 1u);  // 2u << 31 wraps to 0: no later break
        const int end = later ? __ffs(later) - 1 : 32;
        const uint32_t bytes = (uint32_t)(end - lane) * row_bytes;
        const uint64_t pol = l2_evict_first();
        bulk_load(smem_u32(sk + (size_t)t * row_bytes), static_cast<const T *>(a.src_k) + offs[j],
                  bytes, bar, pol);
        bulk_load(smem_u32(sv + (size_t)t * row_bytes), static_cast<const T *>(a.src_v) + offs[j],
                  bytes, bar, pol);
      }
      if (t < PT) s_kind[t] = kinds[j];
    }
  };

  T *dst_k = static_cast<T *>(a.dst_k);
  T *dst_v = static_cast<T *>(a.dst_v);
  const CS *cs = static_cast<const CS *>(a.cos_sin);
  const uint4 zero = make_uint4(0, 0, 0, 0);
  const int rot = a.rotary_dim, half = rot / 2;
  const int krot_vecs = a.vec_rope ? rot / VE : 0;  // K vectors handled by the rotary pass
  const bool copy_k = a.vec_rope || rot == 0;
  constexpr int kDvShift = DV == 8 ? 3 : DV == 16 ? 4 : 5;
  static_assert((1 << kDvShift) == DV, "head_dim / 8 must be 8, 16 or 32");

  if (tid < 32)
    for (int k = 0; k < min(n_mine, kBulkStages); ++k) issue(k);
  __syncthreads();  // the first blocks' kinds are visible
  for (int i = 0; i < n_mine; ++i) {
    const int s = i % kBulkStages;
    const bool got = mbar_wait(bar0 + 8 * s, (i / kBulkStages) & 1);
    if (!__syncthreads_and(got)) {  // CTA-uniform: stop, let the issued copies land, leave
      if (tid == 0) {
        flag_error(a.err, DSB_FLAG_TIMEOUT);
        for (int k = i; k < min(n_mine, i + kBulkStages); ++k)
          mbar_wait(bar0 + 8 * (k % kBulkStages), (k / kBulkStages) & 1);
      }
      return;
    }
    const uint8_t *st = bulk_smem + s * lay.stage;
    const uint8_t *sk = st, *sv = st + lay.v;
    const int *s_kind = reinterpret_cast<const int *>(st + lay.kind);
    const CS *s_cs = reinterpret_cast<const CS *>(st + lay.cs);
    const int64_t p0 = (int64_t)((int)blockIdx.x + i * (int)gridDim.x) << a.pt_shift;
    const int n_tok = (int)min((int64_t)PT, width - p0);
    // element offset of (token t, head h, dim 0) in the destination
    const int64_t dst_base =
        GATHER ? ((int64_t)r * a.working_tokens + p0) * row_elems
               : (slot * heads * (int64_t)a.working_budget + p0) * DH;
    auto dst_off = [&](int t, int h) -> int64_t {
      return GATHER ? dst_base + (int64_t)t * row_elems + h * DH
                    : dst_base + ((int64_t)h * a.working_budget + t) * DH;
    };

    // V, and the K dims past the rotary part: straight copies.  Items run
    // dim-vector fastest, then token, then head (shifts only: PT and DV are
    // powers of two).
    const int n_items = heads << (a.pt_shift + kDvShift);
    for (int it = tid; it < n_items; it += kBulkThreads) {
      const int dv = it & (DV - 1);
      const int t = (it >> kDvShift) & (PT - 1);
      const int h = it >> (kDvShift + a.pt_shift);
      if (t >= n_tok) continue;
      const int kind = s_kind[t];
      if (kind == 0) continue;
      const int64_t o = dst_off(t, h) + dv * VE;
      const size_t so = (size_t)t * row_bytes + ((size_t)h * DH + dv * VE) * 2;
      stg_stream(dst_v + o, kind == 1 ? *reinterpret_cast<const uint4 *>(sv + so) : zero);
      if (copy_k && dv >= krot_vecs)
        stg_stream(dst_k + o, kind == 1 ? *reinterpret_cast<const uint4 *>(sk + so) : zero);
    }

    if (a.vec_rope) {
      // NeoX, half % 8 == 0: item (head, token, j) rotates vectors j and
      // j + half/8 of one head row.  With cs_bulk the cos/sin vectors come
      // from the staged rows; otherwise from the table in global memory.
      const int hv = half / VE;
      const int hv_shift = (hv & (hv - 1)) == 0 ? __ffs(hv) - 1 : -1;
      const int k_items = heads * n_tok * hv;
      for (int it = tid; it < k_items; it += kBulkThreads) {
        const int j = hv_shift >= 0 ? it & (hv - 1) : it % hv;
        const int th = hv_shift >= 0 ? it >> hv_shift : it / hv;  // token + n_tok * head
        const int t = th % n_tok, h = th / n_tok;
        const int kind = s_kind[t];
        if (kind == 0) continue;
        const int64_t o = dst_off(t, h);
        if (kind == 2) {
          stg_stream(dst_k + o + j * VE, zero);
          stg_stream(dst_k + o + half + j * VE, zero);
          continue;
        }
        float c[VE], sn[VE];
        if (a.cs_bulk) {
          const CS *csr = s_cs + (int64_t)t * a.cs_stride;
          cs_load_vec<CS, VE, true>(csr + j * VE, c);
          cs_load_vec<CS, VE, true>(csr + half + j * VE, sn);
        } else {
          const CS *csr = cs + (p0 + t) * a.cs_stride;
          cs_load_vec<CS, VE>(csr + j * VE, c);
          cs_load_vec<CS, VE>(csr + half + j * VE, sn);
        }
        float sneg[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) sneg[e] = -sn[e];
        const uint8_t *hrow = sk + (size_t)t * row_bytes + (size_t)h * DH * 2;
        const uint4 lo = *reinterpret_cast<const uint4 *>(hrow + j * VE * 2);
        const uint4 hi = *reinterpret_cast<const uint4 *>(hrow + (half + j * VE) * 2);
        stg_stream(dst_k + o + j * VE, rotate8<T>(lo, hi, c, sneg));
        stg_stream(dst_k + o + half + j * VE, rotate8<T>(hi, lo, c, sn));
      }
    } else if (rot > 0) {
      // Any other rotary layout: one thread per (token, head, element), the
      // partner element read from the staged row.
      const int n_el = n_tok * heads * DH;
      for (int it = tid; it < n_el; it += kBulkThreads) {
        const int d = it % DH, h = (it / DH) % heads, t = it / (DH * heads);
        const int kind = s_kind[t];
        if (kind == 0) continue;
        T out = Elem<T>::from_f(0.f);
        if (kind == 1) {
          const T *hx = reinterpret_cast<const T *>(sk + (size_t)t * row_bytes) + h * DH;
          if (d >= rot) {
            out = hx[d];
          } else {
            const CS *csr = cs + (p0 + t) * a.cs_stride;
            int ii;
            float x1, x2;
            bool first;
            if (a.neox) {
              first = d < half;
              ii = first ? d : d - half;
              x1 = Elem<T>::to_f(hx[ii]);
              x2 = Elem<T>::to_f(hx[ii + half]);
            } else {
              first = (d & 1) == 0;
              ii = d >> 1;
              x1 = Elem<T>::to_f(hx[2 * ii]);
              x2 = Elem<T>::to_f(hx[2 * ii + 1]);
            }
            const float cc = cs_load(csr + ii), snv = cs_load(csr + half + ii);
            out = Elem<T>::from_f(first ? __fmul_rn(x1, cc) - __fmul_rn(x2, snv)
                                        : __fmul_rn(x2, cc) + __fmul_rn(x1, snv));
          }
        }
        dst_k[dst_off(t, h) + d] = out;
      }
    }
    __syncthreads();  // every thread is done with stage s (and sees the next kinds)
    if (tid < 32 && i + kBulkStages < n_mine) issue(i + kBulkStages);
  }
}

int elem_bytes(int dtype) { return dtype == DSB_F32 ? 4 : 2; }

int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((1LL << s) < v) ++s;
  return s;
}

// DSB_REBUILD_LEGACY=1 selects the cp.async row kernel (kept as the fallback
// for shapes the bulk kernel does not take, and parity-tested on its own).
bool legacy_rope_requested() {
  const char *e = std::getenv("DSB_REBUILD_LEGACY");
  return e != nullptr && e[0] == '1';
}

#ifndef DSB_BULK_STAGE_BYTES
#define DSB_BULK_STAGE_BYTES (32 * 1024)  // K + V rows staged per bulk-kernel CTA
#endif
#ifndef DSB_BULK_PT_MAX
#define DSB_BULK_PT_MAX 64  // positions per stage at most (two per lane of the issuing warp)
#endif
#ifndef DSB_BULK_CS_MAX_BYTES
#define DSB_BULK_CS_MAX_BYTES (16 * 1024)  // cos/sin rows staged per stage at most
#endif

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// CTAs per row for `rows` rows of `nblk` position blocks when `resident`
// CTAs fit on the device at once: a CTA streams per = ceil(nblk / gx) blocks
// through its stages, so it takes about per + 1 block times (the first
// block's copies are not hidden), and a launch takes that many times its
// number of waves.  The smallest such cost wins (fewer CTAs on a tie), so a
// grid never spills a few CTAs into a second wave.
int64_t bulk_ctas_per_row(int64_t rows, int64_t nblk, int64_t resident) {
  resident = std::max<int64_t>(1, resident);
  int64_t best_gx = 1, best_cost = INT64_MAX, best_ctas = INT64_MAX;
  for (int64_t want = 1; want <= nblk; ++want) {
    const int64_t gx = (nblk + want - 1) / want;
    const int64_t per = (nblk + gx - 1) / gx;  // blocks of the busiest CTA
    const int64_t ctas = rows * gx;
    const int64_t cost = ((ctas + resident - 1) / resident) * (per + 1);
    if (cost < best_cost || (cost == best_cost && ctas < best_ctas)) {
      best_cost = cost;
      best_ctas = ctas;
      best_gx = gx;
    }
  }
  return best_gx;
}

// The bulk kernel when its preconditions hold: 16-bit caches, head_dim 64,
// 128 or 256, 16-byte aligned bases and at least one K+V row pair per stage.
template <typename T, typename CS, bool GATHER>
int launch_rope_bulk(RopeArgs a, int rows, int64_t width, cudaStream_t st) {
  if constexpr (sizeof(T) != 2) {
    return -1;
  } else {
    if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return -1;
    if (!aligned16(a.src_k) || !aligned16(a.src_v) || !aligned16(a.dst_k) || !aligned16(a.dst_v))
      return -1;
    const int64_t row_bytes = (int64_t)a.heads * a.head_dim * 2;
    int pt = DSB_BULK_PT_MAX;  // two positions per lane of the issuing warp at most
    while (pt > 1 && 2 * pt * row_bytes > DSB_BULK_STAGE_BYTES) pt >>= 1;
    if (2 * pt * row_bytes > DSB_BULK_STAGE_BYTES) return -1;
    a.chunk_shift = log2_exact(a.chunk);
    a.block_shift = log2_exact(a.block_size);
    constexpr int VE = 8;
    a.vec_rope = a.neox && a.rotary_dim > 0 && (a.rotary_dim / 2) % VE == 0 &&
                 reinterpret_cast<uintptr_t>(a.cos_sin) % 16 == 0 &&
                 (a.cs_stride * (int64_t)sizeof(CS)) % 16 == 0;
    auto kern = a.head_dim == 128  ? rope_bulk_kernel<T, CS, GATHER, 128>
                : a.head_dim == 64 ? rope_bulk_kernel<T, CS, GATHER, 64>
                                   : rope_bulk_kernel<T, CS, GATHER, 256>;
    // Stage the cos/sin rows with the K/V rows when the table is dense (row
    // stride = rotary_dim, so the CTA's rows are one contiguous range that
    // ends inside the table) and they take at most 16 KB per CTA.
    const int64_t cs_row_bytes = a.cs_stride * (int64_t)sizeof(CS);
    auto stage_smem = [&](int p, int &cs_bulk) {
      cs_bulk = a.vec_rope && a.cs_stride == a.rotary_dim && p * cs_row_bytes <= DSB_BULK_CS_MAX_BYTES;
      return bulk_smem_layout(p, row_bytes, GATHER ? 0 : a.plan_width - 5, cs_bulk ? p * cs_row_bytes : 0)
          .total;
    };
    // The largest block (up to 32 KB of K + V rows) at which kBulkMinCtas
    // CTAs stay resident per SM.  Measured at config 2's lengths (µs per
    // launch; rows x kv heads of 128): 16 x 4 takes 16 positions (22.7),
    // 32 x 2 16 (22.8; 32 positions leave 2 CTAs per SM: 24.5), 64 x 1 32
    // (23.1; 64 positions with their cos/sin rows leave 2 per SM: 28.2).
    constexpr int kBulkMinCtas = 3;
    const int sms = std::max(1, sm_count());
    int cs_bulk = 0;
    size_t smem = stage_smem(pt, cs_bulk);
    for (int p = pt; p >= 1; p >>= 1) {
      int csb = 0;
      const size_t sm_p = stage_smem(p, csb);
      if (int e = ensure_smem((const void *)kern, sm_p); e != DSB_OK) return e;
      if (resident_ctas((const void *)kern, kBulkThreads, sm_p) >= kBulkMinCtas * sms) {
        pt = p;
        smem = sm_p;
        cs_bulk = csb;
        break;
      }
    }
    a.pt_shift = log2_exact(pt);
    a.cs_bulk = cs_bulk;
    if (int e = ensure_smem((const void *)kern, smem); e != DSB_OK) return e;
    // Each CTA streams an equal share of its row's position blocks; the
    // share is picked against the resident CTA count (bulk_ctas_per_row).
    const int64_t nblk = (width + pt - 1) / pt;
    const int64_t gx =
        bulk_ctas_per_row(rows, nblk, resident_ctas((const void *)kern, kBulkThreads, smem));
    if (gx > 0x7fffffff || rows > 65535) return fail(DSB_ERR_UNSUPPORTED, "grid too large");
    launch_kernel(kern, dim3((unsigned)gx, rows), dim3(kBulkThreads), smem, st, a);
    return check_launch(GATHER ? "gather_rope_bulk_kernel" : "rebuild_rope_bulk_kernel");
  }
}

// -1: no kernel of this build takes the launch (only for a rebuild from the
// selection state, which the caller then runs as plan + rebuild).
template <typename T, typename CS, bool GATHER>
int launch_rope(RopeArgs a, int rows, int64_t width, cudaStream_t st) {
  if (!legacy_rope_requested()) {
    const int e = launch_rope_bulk<T, CS, GATHER>(a, rows, width, st);
    if (e >= 0) return e;
  }
  if (a.from_sel) return -1;
  const int row_bytes = a.heads * a.head_dim * (int)sizeof(T);
  int U = row_bytes <= 1024 ? 2 : 1;
  const size_t smem = (size_t)kWarpsRope * 2 * U * 2 * row_bytes;  // double-buffered K+V rows
  if (smem > 200 * 1024) return fail(DSB_ERR_UNSUPPORTED, "KV rows too wide for staging");
  a.tokens_per_warp = U;
  constexpr int VE = 16 / (int)sizeof(T);
  a.vec_rope = a.neox && a.rotary_dim > 0 && (a.rotary_dim / 2) % VE == 0 &&
               reinterpret_cast<uintptr_t>(a.cos_sin) % 16 == 0 &&
               (a.cs_stride * (int64_t)sizeof(CS)) % 16 == 0;
  a.chunk_shift = log2_exact(a.chunk);
  a.block_shift = log2_exact(a.block_size);
  auto kern = a.head_dim == 128   ? rope_rows_kernel<T, CS, GATHER, 128>
              : a.head_dim == 64  ? rope_rows_kernel<T, CS, GATHER, 64>
              : a.head_dim == 256 ? rope_rows_kernel<T, CS, GATHER, 256>
                                  : rope_rows_kernel<T, CS, GATHER, 0>;
  if (int st_ = ensure_smem((const void *)kern, smem); st_ != DSB_OK) return st_;
  const int64_t per_cta = (int64_t)kWarpsRope * U;
  // enough CTAs to fill the GPU once; each warp then loops over its batches
  int resident = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, kWarpsRope * 32, smem) !=
          cudaSuccess || resident <= 0)
    resident = 1;
  const int64_t fill = ((int64_t)resident * sm_count() + rows - 1) / rows;
  const int64_t gx = std::max<int64_t>(1, std::min<int64_t>((width + per_cta - 1) / per_cta, fill));
  if (gx > 0x7fffffff || rows > 65535) return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  launch_kernel(kern, dim3((unsigned)gx, rows), dim3(kWarpsRope * 32), smem, st, a);
  return check_launch(GATHER ? "gather_rope_kernel" : "rebuild_rope_kernel");
}

template <bool GATHER>
int dispatch_rope(const RopeArgs &a, int dtype, int cs_dtype, int rows, int64_t width,
                  cudaStream_t st) {
#define DSB_RP(TD, T, CD, CS) \
  if (dtype == TD && cs_dtype == CD) return launch_rope<T, CS, GATHER>(a, rows, width, st);
  DSB_RP(DSB_BF16, __nv_bfloat16, DSB_BF16, __nv_bfloat16)
  DSB_RP(DSB_BF16, __nv_bfloat16, DSB_F32, float)
  DSB_RP(DSB_BF16, __nv_bfloat16, DSB_F16, __half)
  DSB_RP(DSB_F16, __half, DSB_F16, __half)
  DSB_RP(DSB_F16, __half, DSB_F32, float)
  DSB_RP(DSB_F16, __half, DSB_BF16, __nv_bfloat16)
  DSB_RP(DSB_F32, float, DSB_F32, float)
  DSB_RP(DSB_F32, float, DSB_BF16, __nv_bfloat16)
  DSB_RP(DSB_F32, float, DSB_F16, __half)
#undef DSB_RP
  return fail(DSB_ERR_INVALID, "unknown dtype");
}

int common_checks(int heads, int head_dim, int rotary_dim, int dtype) {
  if (heads <= 0 || head_dim <= 0)
    return fail(DSB_ERR_INVALID, "raw sequence, head and head dimensions must be positive");
  if (rotary_dim < 0 || rotary_dim > head_dim || rotary_dim % 2)
    return fail(DSB_ERR_INVALID, "rotary_dim must be even and between zero and head_dim");
  if (dtype != DSB_BF16 && dtype != DSB_F16 && dtype != DSB_F32)
    return fail(DSB_ERR_INVALID, "KV caches must use BF16, FP16 or FP32");
  if ((head_dim * elem_bytes(dtype)) % 16)
    return fail(DSB_ERR_UNSUPPORTED, "head_dim * element size must be a multiple of 16 bytes");
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_rebuild_compact_kv_from_plan(
    const void *raw_key, const void *raw_value, void *working_key, void *working_value,
    const int64_t *plan, int32_t plan_rows, int32_t plan_width, const void *cos_sin_cache,
    int32_t cos_sin_dtype, int64_t cos_sin_stride, int64_t cos_sin_rows, int32_t num_slots,
    int64_t max_model_len, int32_t num_heads, int32_t head_dim, int32_t working_budget,
    int32_t chunk_size, int32_t max_width, int32_t rotary_dim, int32_t is_neox_style,
    int32_t dtype, int32_t *error_flag, void *stream) {
  int c = common_checks(num_heads, head_dim, rotary_dim, dtype);
  if (c != DSB_OK) return c;
  if (max_model_len <= 0 || num_slots <= 0)
    return fail(DSB_ERR_INVALID, "raw sequence, head and head dimensions must be positive");
  if (plan_rows < 0 || plan_rows > num_slots || max_width < 0 || max_width > working_budget)
    return fail(DSB_ERR_INVALID, "KV plan exceeds the working cache batch or token capacity");
  if (chunk_size <= 0 || plan_width != 5 + working_budget / chunk_size)
    return fail(DSB_ERR_INVALID, "plan width must be 5 + working_budget // chunk_size");
  if (rotary_dim > 0 && (cos_sin_rows < max_width || cos_sin_stride < rotary_dim))
    return fail(DSB_ERR_INVALID, "cos/sin cache must contain all local positions and rotary dimensions");
  if (plan_rows == 0 || max_width == 0) return DSB_OK;
  if (!raw_key || !raw_value || !working_key || !working_value || !plan ||
      (rotary_dim > 0 && !cos_sin_cache))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  RopeArgs a{};
  a.src_k = raw_key;
  a.src_v = raw_value;
  a.dst_k = working_key;
  a.dst_v = working_value;
  a.plan = plan;
  a.plan_width = plan_width;
  a.num_slots = num_slots;
  a.max_model_len = max_model_len;
  a.working_budget = working_budget;
  a.chunk = chunk_size;
  a.max_width = max_width;
  a.cos_sin = cos_sin_cache;
  a.cs_stride = cos_sin_stride;
  a.cs_rows = cos_sin_rows;
  a.heads = num_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.neox = is_neox_style ? 1 : 0;
  a.err = error_flag;
  return dispatch_rope<false>(a, dtype, rotary_dim > 0 ? cos_sin_dtype : DSB_F32, plan_rows,
                              max_width, as_stream(stream));
}

extern "C" int dsb_rebuild_working_cache(
    const void *raw_key, const void *raw_value, void *working_key, void *working_value,
    const int32_t *row_slots, const int32_t *committed_lens, int32_t rows,
    const int32_t *sel_chunks, int32_t sel_stride, const int32_t *sel_count, int32_t num_slots,
    int32_t chunk_size, int32_t history_budget, int32_t recent_window, int32_t plan_width,
    int64_t *plan, int32_t *history_lens, int32_t *working_lens, const void *cos_sin_cache,
    int32_t cos_sin_dtype, int64_t cos_sin_stride, int64_t cos_sin_rows, int64_t max_model_len,
    int32_t num_heads, int32_t head_dim, int32_t working_budget, int32_t rotary_dim,
    int32_t is_neox_style, int32_t dtype, int32_t *error_flag, void *stream) {
  int c = common_checks(num_heads, head_dim, rotary_dim, dtype);
  if (c != DSB_OK) return c;
  if (rows < 0) return fail(DSB_ERR_INVALID, "negative rows");
  if (rows == 0) return DSB_OK;
  if (max_model_len <= 0 || num_slots <= 0)
    return fail(DSB_ERR_INVALID, "raw sequence, head and head dimensions must be positive");
  if (chunk_size <= 0 || history_budget <= 0 || sel_stride <= 0)
    return fail(DSB_ERR_INVALID, "bad chunk size, budget, plan width or selection stride");
  if (recent_window == 0) recent_window = chunk_size;
  if (recent_window < chunk_size || recent_window % chunk_size || recent_window > history_budget)
    return fail(DSB_ERR_INVALID,
                "recent_window must be a chunk-size multiple in [chunk_size, history_budget]");
  if (rows > num_slots || history_budget > working_budget)
    return fail(DSB_ERR_INVALID, "KV plan exceeds the working cache batch or token capacity");
  if (plan_width != 5 + working_budget / chunk_size)
    return fail(DSB_ERR_INVALID, "plan width must be 5 + working_budget // chunk_size");
  if (rotary_dim > 0 && (cos_sin_rows < history_budget || cos_sin_stride < rotary_dim))
    return fail(DSB_ERR_INVALID, "cos/sin cache must contain all local positions and rotary dimensions");
  if (!raw_key || !raw_value || !working_key || !working_value || !committed_lens ||
      !sel_chunks || !sel_count || (rotary_dim > 0 && !cos_sin_cache))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  RopeArgs a{};
  a.src_k = raw_key;
  a.src_v = raw_value;
  a.dst_k = working_key;
  a.dst_v = working_value;
  a.plan_width = plan_width;
  a.num_slots = num_slots;
  a.max_model_len = max_model_len;
  a.working_budget = working_budget;
  a.chunk = chunk_size;
  a.max_width = history_budget;
  a.cos_sin = cos_sin_cache;
  a.cs_stride = cos_sin_stride;
  a.cs_rows = cos_sin_rows;
  a.heads = num_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.neox = is_neox_style ? 1 : 0;
  a.err = error_flag;
  a.from_sel = 1;
  a.row_slots = row_slots;
  a.committed_lens = committed_lens;
  a.sel_chunks = sel_chunks;
  a.sel_count = sel_count;
  a.sel_stride = sel_stride;
  a.history_budget = history_budget;
  a.window = recent_window;
  a.plan_out = plan;
  a.hist_out = history_lens;
  a.wlen_out = working_lens;
  const int e = dispatch_rope<false>(a, dtype, rotary_dim > 0 ? cos_sin_dtype : DSB_F32, rows,
                                     history_budget, as_stream(stream));
  if (e != -1) return e;
  // No fused kernel for this shape (or the row kernel was requested): plan,
  // then rebuild from it.
  if (plan == nullptr)
    return fail(DSB_ERR_UNSUPPORTED, "this cache layout needs a plan buffer (two-launch path)");
  c = dsb_build_history_plan(row_slots, committed_lens, rows, sel_chunks, sel_stride, sel_count,
                             num_slots, chunk_size, history_budget, recent_window, plan_width,
                             plan, history_lens, working_lens, error_flag, stream);
  if (c != DSB_OK) return c;
  return dsb_rebuild_compact_kv_from_plan(raw_key, raw_value, working_key, working_value, plan,
                                          rows, plan_width, cos_sin_cache, cos_sin_dtype,
                                          cos_sin_stride, cos_sin_rows, num_slots, max_model_len,
                                          num_heads, head_dim, working_budget, chunk_size,
                                          history_budget, rotary_dim, is_neox_style, dtype,
                                          error_flag, stream);
}

extern "C" int dsb_gather_raw_kv_with_local_rope(
    const void *raw_key_cache, const void *raw_value_cache, int64_t num_blocks,
    int32_t block_size, int32_t num_heads, int32_t head_dim, const int32_t *block_table,
    int64_t block_table_stride, int64_t block_table_cols,
    const int64_t *selected_token_indices, int32_t batch, int32_t working_tokens,
    const void *cos_sin_cache, int32_t cos_sin_dtype, int64_t cos_sin_stride,
    int64_t cos_sin_rows, int32_t rotary_dim, int32_t is_neox_style, int32_t dtype,
    void *out_key, void *out_value, int32_t *error_flag, void *stream) {
  int c = common_checks(num_heads, head_dim, rotary_dim, dtype);
  if (c != DSB_OK) return c;
  if (batch < 0 || working_tokens < 0) return fail(DSB_ERR_INVALID, "negative sizes");
  if (batch == 0 || working_tokens == 0) return DSB_OK;
  if (num_blocks <= 0 || block_size <= 0 || block_table_cols <= 0)
    return fail(DSB_ERR_INVALID, "block table and cache must be non-empty");
  if (rotary_dim > 0 && (cos_sin_rows < working_tokens || cos_sin_stride < rotary_dim))
    return fail(DSB_ERR_INVALID, "cos/sin cache must contain all local positions and rotary dimensions");
  if (!raw_key_cache || !raw_value_cache || !block_table || !selected_token_indices ||
      !out_key || !out_value || (rotary_dim > 0 && !cos_sin_cache))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  RopeArgs a{};
  a.src_k = raw_key_cache;
  a.src_v = raw_value_cache;
  a.dst_k = out_key;
  a.dst_v = out_value;
  a.bt = block_table;
  a.bt_stride = block_table_stride;
  a.bt_cols = block_table_cols;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.sel = selected_token_indices;
  a.working_tokens = working_tokens;
  a.cos_sin = cos_sin_cache;
  a.cs_stride = cos_sin_stride;
  a.cs_rows = cos_sin_rows;
  a.heads = num_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.neox = is_neox_style ? 1 : 0;
  a.err = error_flag;
  return dispatch_rope<true>(a, dtype, rotary_dim > 0 ? cos_sin_dtype : DSB_F32, batch,
                             working_tokens, as_stream(stream));
}
