"""One Eagle3-style draft decoder layer over the DiffSpec draft cache.

The draft model of diffspec runs one decoder layer per draft step: its qkv
projection takes the token embedding concatenated with the target's hidden
state (diffspec/vllm_patch.py:189-225), the sink op hands the pre-RoPE K/V
to the canonical cache (vllm_patch.py:132-178, runtime.py:1602-1618), RoPE is
applied at the working cache's local positions (runtime.py:1767-1794), and
the attention runs over the compact working cache (runtime.py:2024-2134),
followed by the output projection and a SwiGLU MLP with RMSNorm.

Every stage is this library's kernels: RMSNorm, the query + K/V projection
with the raw-cache write (one tcgen05 launch), RoPE of q/k, the draft
attention, and the output / gate-up / down projections on the same
weight-streaming tcgen05 linear kernel with the residual adds and SwiGLU in
its epilogue.  The
weights are random (no checkpoint is involved); the layer exists to turn the
kernels into draft tokens per second and to show how the
pieces compose.  The LM head is not included: its vocabulary is unspecified.
"""

from __future__ import annotations

import torch

from . import _lib
from .attention import AttentionWorkspace, draft_decode_attention
from .kernels import qkv_projection_write_raw

__all__ = ["Eagle3DraftLayer", "Eagle3DraftLayerTP", "add_rms_norm", "draft_linear",
           "draft_linear_peer", "peer_add_rms_norm",
           "interleave_gate_up", "pack_linear_weight", "rms_norm", "rope_qk", "silu_mul"]


def _rows(t: torch.Tensor, what: str) -> int:
    """Row stride (elements) of a 2-D tensor with unit column stride."""
    if t.ndim != 2 or t.stride(1) != 1:
        raise ValueError(f"{what} must be 2-D with contiguous rows")
    return t.stride(0)


_EPILOGUES = {"plain": 0, "residual": 1, "swiglu": 2, "partial": 3}


def interleave_gate_up(weight: torch.Tensor) -> torch.Tensor:
    """A ``[2 * inter, K]`` gate_up weight (gate rows, then up rows) in the
    tile order ``draft_linear(..., "swiglu")`` reads: 128-row tiles whose
    first 64 rows are gate rows ``64 i .. 64 i + 63`` and last 64 the
    matching up rows.  A one-time permutation at load time."""
    inter = weight.shape[0] // 2
    if weight.shape[0] != 2 * inter or inter % 64:
        raise ValueError("gate_up weight rows must be 2 * inter with inter a multiple of 64")
    gate, up = weight[:inter].view(inter // 64, 64, -1), weight[inter:].view(inter // 64, 64, -1)
    return torch.stack((gate, up), 1).reshape(2 * inter, -1).contiguous()


def pack_linear_weight(weight: torch.Tensor) -> torch.Tensor:
    """A ``[rows, K]`` weight (rows a multiple of 128, K of 64) in the
    tile-packed layout that ``draft_linear(..., packed=True)`` streams: every
    128-row x 64-column block the kernel loads becomes one contiguous 16 KB
    run in the 128-byte-swizzled order of the tensor cores' shared-memory
    operand (row r's 16-byte piece p at position p ^ (r % 8)), so the kernel
    stages it with one bulk copy.  One launch (``dsb_pack_linear_weight``),
    done once at load time; the result has the same bytes, reordered."""
    if weight.ndim != 2 or weight.shape[0] % 128 or weight.shape[1] % 64:
        raise ValueError("weight must be [rows, K] with rows % 128 == 0 and K % 64 == 0")
    device = _lib.require_cuda(weight)
    weight = weight.contiguous()
    out = torch.empty_like(weight)
    _lib.call("dsb_pack_linear_weight", _lib.ptr(weight), weight.shape[0], weight.shape[1],
              _lib.dtype_code(weight.dtype), _lib.ptr(out), _lib.stream_ptr(device))
    return out


def draft_linear(x: torch.Tensor, weight: torch.Tensor, epilogue: str = "plain",
                 residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 prefetch_weight: bool = True, packed: bool = False,
                 prefetch_l2: bool = False) -> torch.Tensor:
    """``x [T, K] @ weight.T`` on the tensor cores (``dsb_draft_linear``),
    with ``epilogue`` "plain", "residual" (``+ residual`` before the one
    rounding), "partial" (the fp32 sums unrounded, ``out`` float32: one
    rank's share of a row-split linear) or "swiglu" (``weight`` from :func:`interleave_gate_up`; out
    ``[T, rows / 2] = round(round(silu(gate)) * up)`` with gate and up
    rounded first, as vLLM's gate_up output and SiluAndMul round them).  ``prefetch_weight`` starts the
    weight stream before the previous kernel has finished (the weight must
    not be written by that kernel); ``prefetch_l2`` also requests the next
    weight blocks of every CTA into L2 by then (faster alone; it puts more
    of the weight in L2).
    ``packed``: ``weight`` comes from :func:`pack_linear_weight` (same shape,
    tile-packed bytes)."""
    if epilogue not in _EPILOGUES:
        raise ValueError(f"epilogue must be one of {sorted(_EPILOGUES)}")
    if x.ndim != 2 or weight.ndim != 2 or weight.shape[1] != x.shape[1] or x.dtype != weight.dtype:
        raise ValueError("x must be [T, K] and weight [rows, K] in one dtype")
    if not (x.is_contiguous() and weight.is_contiguous()):
        raise ValueError("x and weight must be contiguous")
    cols = weight.shape[0] // 2 if epilogue == "swiglu" else weight.shape[0]
    device = _lib.require_cuda(x, weight, residual, out)
    if epilogue == "residual":
        if residual is None or residual.shape != (x.shape[0], cols) or residual.dtype != x.dtype:
            raise ValueError("residual must be [T, rows] in the input dtype")
        res_stride = _rows(residual, "residual")
    else:
        res_stride = 0
    out_dtype = torch.float32 if epilogue == "partial" else x.dtype
    if out is None:
        out = torch.empty((x.shape[0], cols), dtype=out_dtype, device=device)
    elif out.shape != (x.shape[0], cols) or out.dtype != out_dtype:
        raise ValueError("out has the wrong shape or dtype")
    _lib.call("dsb_draft_linear", _lib.ptr(x), x.shape[0], x.shape[1], _lib.ptr(weight),
              weight.shape[0], _EPILOGUES[epilogue], _lib.ptr(residual), res_stride, _lib.ptr(out),
              _rows(out, "out"), _lib.dtype_code(x.dtype),
              (1 if prefetch_weight else 0) | (2 if packed else 0) | (4 if prefetch_l2 else 0),
              _lib.ptr(_lib.error_flag(device)), _lib.stream_ptr(device))
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """``round(round(x * rsqrt(mean(x^2) + eps)) * weight)`` per row of ``x
    [rows, cols]`` (fp32 math, rounded where vLLM's rms_norm rounds), one
    launch (``dsb_rms_norm``)."""
    if weight.shape != (x.shape[-1],) or weight.dtype != x.dtype:
        raise ValueError("weight must be [cols] in the rows' dtype")
    device = _lib.require_cuda(x, weight, out)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=device)
    elif out.shape != x.shape or out.dtype != x.dtype:
        raise ValueError("out must match x")
    _lib.call("dsb_rms_norm", _lib.ptr(x), _rows(x, "x"), _lib.ptr(weight.contiguous()),
              _lib.ptr(out), _rows(out, "out"), x.shape[0], x.shape[1], float(eps),
              _lib.dtype_code(x.dtype), _lib.stream_ptr(device))
    return out


def add_rms_norm(partial: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor | None,
                 eps: float, x_out: torch.Tensor | None = None,
                 out: torch.Tensor | None = None):
    """``x = round(partial + residual)`` (fp32 ``partial [rows, cols]``, e.g.
    an all-reduced "partial" linear, one rounding) and, when ``weight`` is
    given, ``rms_norm(x)`` with :func:`rms_norm`'s arithmetic bit for bit;
    one launch (``dsb_add_rms_norm``).  Returns ``(x, normed)`` (``normed``
    None without a weight)."""
    if partial.dtype != torch.float32 or partial.shape != residual.shape:
        raise ValueError("partial must be fp32 and shaped like residual")
    if weight is not None and (weight.shape != (residual.shape[-1],) or weight.dtype != residual.dtype):
        raise ValueError("weight must be [cols] in the residual's dtype")
    device = _lib.require_cuda(partial, residual, weight, x_out, out)
    if x_out is None:
        x_out = torch.empty_like(residual)
    if weight is not None and out is None:
        out = torch.empty_like(residual)
    _lib.call("dsb_add_rms_norm", _lib.ptr(partial), _rows(partial, "partial"), _lib.ptr(residual),
              _rows(residual, "residual"), _lib.ptr(weight), _lib.ptr(x_out), _rows(x_out, "x_out"),
              _lib.ptr(out), _rows(out, "out") if out is not None else 0, residual.shape[0],
              residual.shape[1], float(eps), _lib.dtype_code(residual.dtype),
              _lib.stream_ptr(device))
    return x_out, out


def draft_linear_peer(x: torch.Tensor, weight: torch.Tensor, site, packed: bool = False,
                      prefetch_weight: bool = True) -> None:
    """This rank's share of a row-split linear, all-reduced over NVLink:
    ``x [T, K] @ weight.T`` as :func:`draft_linear` computes it, its fp32 sums
    stored into this rank's slot of every rank's exchange buffer of ``site``
    (a :class:`parallel.PeerExchange`), one launch
    (``dsb_draft_linear_peer``).  Read the reduced result with
    :func:`peer_add_rms_norm`."""
    if x.ndim != 2 or weight.ndim != 2 or weight.shape[1] != x.shape[1] or x.dtype != weight.dtype:
        raise ValueError("x must be [T, K] and weight [rows, K] in one dtype")
    if not (x.is_contiguous() and weight.is_contiguous()):
        raise ValueError("x and weight must be contiguous")
    if weight.shape[0] != site.features or x.shape[0] > site.tokens_max:
        raise ValueError("weight rows must equal the site's features and T its token capacity")
    device = _lib.require_cuda(x, weight)
    _lib.call("dsb_draft_linear_peer", _lib.ptr(x), x.shape[0], x.shape[1], _lib.ptr(weight),
              weight.shape[0], _lib.ptr(site.bases), site.world, site.rank, site.tokens_max,
              site.own_base, _lib.dtype_code(x.dtype),
              (1 if prefetch_weight else 0) | (2 if packed else 0),
              _lib.ptr(_lib.error_flag(device)), _lib.stream_ptr(device))


def peer_add_rms_norm(site, residual: torch.Tensor, weight: torch.Tensor | None, eps: float,
                      x_out: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """:func:`add_rms_norm` whose fp32 ``partial`` is the sum, in rank order,
    of every rank's :func:`draft_linear_peer` partial of ``site``'s current
    call, once all of them have arrived (``dsb_peer_add_rms_norm``; a wait
    bounded by time, after which the error word carries
    DSB_FLAG_TIMEOUT).  Returns ``(x, normed)``."""
    if residual.ndim != 2 or residual.shape[1] != site.features or residual.shape[0] > site.tokens_max:
        raise ValueError("residual must be [T <= tokens_max, features]")
    if weight is not None and (weight.shape != (residual.shape[-1],) or weight.dtype != residual.dtype):
        raise ValueError("weight must be [cols] in the residual's dtype")
    device = _lib.require_cuda(residual, weight, x_out, out)
    if x_out is None:
        x_out = torch.empty_like(residual)
    if weight is not None and out is None:
        out = torch.empty_like(residual)
    _lib.call("dsb_peer_add_rms_norm", site.own_base, site.world, site.tokens_max,
              _lib.ptr(residual), _rows(residual, "residual"), _lib.ptr(weight), _lib.ptr(x_out),
              _rows(x_out, "x_out"), _lib.ptr(out), _rows(out, "out") if out is not None else 0,
              residual.shape[0], residual.shape[1], float(eps), _lib.dtype_code(residual.dtype),
              _lib.ptr(_lib.error_flag(device)), _lib.stream_ptr(device))
    return x_out, out


def rope_qk(query: torch.Tensor, kv: torch.Tensor, positions: torch.Tensor,
            cos_sin: torch.Tensor, num_kv_heads: int,
            key_out: torch.Tensor | None = None, value_out: torch.Tensor | None = None,
            position_offset: int = 0):
    """NeoX RoPE of one step at ``positions [T] + position_offset`` (int32) of
    a ``[rows, cos | sin]`` table: ``query [T, Hq * D]`` is rotated in place; the K half of
    the packed K/V projection rows ``kv [T, 2 * Hk * D]`` is rotated into
    ``key_out [T, Hk, D]`` and its V half copied into ``value_out``, the
    contiguous rows the draft attention reads.  One launch
    (``dsb_rope_qk``); returns ``(key_out, value_out)``."""
    tokens = query.shape[0]
    feats = kv.shape[1] // 2
    d = feats // num_kv_heads
    if kv.shape[0] != tokens or kv.shape[1] != 2 * num_kv_heads * d or query.shape[1] % d:
        raise ValueError("query must be [T, Hq * D] and kv [T, 2 * Hk * D]")
    if not (query.dtype == kv.dtype) or cos_sin.ndim != 2 or cos_sin.stride(1) != 1:
        raise ValueError("query and kv share a dtype; cos_sin is a [rows, D] table")
    if positions.dtype != torch.int32 or positions.numel() < tokens:
        raise ValueError("positions must be int32 with one entry per token")
    device = _lib.require_cuda(query, kv, positions, cos_sin, key_out, value_out)
    shape = (tokens, num_kv_heads, d)
    for name, t in (("key_out", key_out), ("value_out", value_out)):
        if t is not None and (t.shape != shape or t.dtype != kv.dtype or not t.is_contiguous()):
            raise ValueError(f"{name} must be contiguous [T, Hk, D] in the kv dtype")
    if key_out is None:
        key_out = torch.empty(shape, dtype=kv.dtype, device=device)
    if value_out is None:
        value_out = torch.empty(shape, dtype=kv.dtype, device=device)
    kv_stride = _rows(kv, "kv")
    _lib.call("dsb_rope_qk", _lib.ptr(query), _rows(query, "query"), query.shape[1] // d,
              _lib.ptr(kv), kv_stride, _lib.ptr(key_out), kv.data_ptr() + feats * kv.element_size(),
              kv_stride, _lib.ptr(value_out), num_kv_heads, d, _lib.ptr(positions),
              int(position_offset), tokens,
              _lib.ptr(cos_sin), cos_sin.stride(0), cos_sin.shape[0],
              _lib.dtype_code(cos_sin.dtype), _lib.dtype_code(kv.dtype),
              _lib.ptr(_lib.error_flag(device)), _lib.stream_ptr(device))
    return key_out, value_out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU ``round(round(silu(gate)) * up)`` of ``gate_up [rows, 2 *
    inter]`` (gate columns first, fp32 math rounded where vLLM's SiluAndMul
    rounds), one launch (``dsb_silu_mul``)."""
    rows, two_inter = gate_up.shape
    inter = two_inter // 2
    device = _lib.require_cuda(gate_up, out)
    if out is None:
        out = torch.empty((rows, inter), dtype=gate_up.dtype, device=device)
    elif out.shape != (rows, inter) or out.dtype != gate_up.dtype:
        raise ValueError("out must be [rows, inter] in the input dtype")
    _lib.call("dsb_silu_mul", _lib.ptr(gate_up), _rows(gate_up, "gate_up"), _lib.ptr(out),
              _rows(out, "out"), rows, inter, _lib.dtype_code(gate_up.dtype),
              _lib.stream_ptr(device))
    return out


class Eagle3DraftLayer:
    """Random-init weights of one draft layer (bf16): hidden 2048, qkv input
    4096 (embedding + hidden), 32 query / 4 kv heads of 128, SwiGLU 6144."""

    def __init__(self, device, *, hidden=2048, qkv_in=4096, num_heads=32, num_kv_heads=4,
                 head_dim=128, intermediate=6144, dtype=torch.bfloat16, seed=0, eps=1e-6):
        g = torch.Generator(device=device).manual_seed(seed)

        def w(rows, cols):
            return (torch.randn((rows, cols), generator=g, device=device) / cols ** 0.5).to(dtype)

        self.hq, self.hk, self.d, self.eps = num_heads, num_kv_heads, head_dim, eps
        self.inter = intermediate
        # one [q | K | V] weight for the fused projection; w_q / w_kv are views
        self.w_qkv = w((num_heads + 2 * num_kv_heads) * head_dim, qkv_in)
        self.w_q = self.w_qkv[: num_heads * head_dim]
        self.w_kv = self.w_qkv[num_heads * head_dim:]  # K rows, then V rows
        self.w_o = w(hidden, num_heads * head_dim)
        self.w_gate_up = w(2 * intermediate, hidden)
        self.w_down = w(hidden, intermediate)
        # the gate/up weight in the tile order of the SwiGLU epilogue (a
        # one-time permutation; w_gate_up keeps the [gate | up] order)
        self.w_gate_up_tiles = interleave_gate_up(self.w_gate_up)
        # what step() streams: every weight tile-packed once (same bytes,
        # reordered so each 128 x 64 block the kernel loads is contiguous)
        self.p_qkv = pack_linear_weight(self.w_qkv)
        self.p_o = pack_linear_weight(self.w_o)
        self.p_gate_up = pack_linear_weight(self.w_gate_up_tiles)
        self.p_down = pack_linear_weight(self.w_down)
        self.in_norm = torch.ones(qkv_in, dtype=dtype, device=device)
        self.post_norm = torch.ones(hidden, dtype=dtype, device=device)
        self.workspace = AttentionWorkspace(device)
        # linears ("qkv", "o_proj", "gate_up", "down_proj") whose whole weight
        # is requested into L2 while the kernel before them runs
        self.l2_prefetch: frozenset[str] = frozenset()

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for t in (self.w_q, self.w_kv, self.w_o, self.w_gate_up, self.w_down))

    def step(self, x_in, residual, *, slots, abs_positions, local_positions, raw_key, raw_value,
             working_key, working_value, cos_sin, out=None, position_offset=0):
        """One draft step for ``n`` rows: ``x_in [n, qkv_in]`` (embedding +
        hidden), ``residual [n, hidden]``.  Writes this step's pre-RoPE K/V to
        the raw caches at ``[slots, abs_positions]`` and its RoPE'd K/V into
        the working caches at ``local_positions + position_offset`` (step j
        of a cycle passes the plan's history lengths and j); returns the
        layer output ``[n, hidden]``."""
        n = x_in.shape[0]
        h = rms_norm(x_in, self.in_norm, self.eps)
        l2 = self.l2_prefetch
        q, kv = qkv_projection_write_raw(h, self.p_qkv, self.hq * self.d, slots, abs_positions,
                                         raw_key, raw_value, prefetch_weight=True,
                                         packed_weight=True, prefetch_l2="qkv" in l2)
        k, v = rope_qk(q, kv, local_positions, cos_sin, self.hk, position_offset=position_offset)
        attn = draft_decode_attention(q.view(n, self.hq, self.d), k, v, working_key, working_value,
                                      slots, local_positions, self.d ** -0.5,
                                      position_offset=position_offset, workspace=self.workspace)
        x = draft_linear(attn.view(n, self.hq * self.d), self.p_o, "residual", residual,
                         packed=True, prefetch_l2="o_proj" in l2)
        act = draft_linear(rms_norm(x, self.post_norm, self.eps), self.p_gate_up, "swiglu",
                           packed=True, prefetch_l2="gate_up" in l2)
        return draft_linear(act, self.p_down, "residual", x, out=out, packed=True,
                            prefetch_l2="down_proj" in l2)


class Eagle3DraftLayerTP:
    """One tensor-parallel shard of an :class:`Eagle3DraftLayer` on rank
    ``rank`` of ``world`` (vLLM's tensor-parallel split of the Eagle3 layer:
    QKVParallelLinear / MergedColumnParallelLinear column-split,
    RowParallelLinear row-split):

    * query heads ``[rank * Hq / world, (rank + 1) * Hq / world)`` and the kv
      heads they read: ``Hk / world`` of them when ``world <= Hk``, else one
      kv head replicated on ``world / Hk`` ranks;
    * qkv and gate_up column-split (this rank's heads and ``inter / world``
      SwiGLU features), o_proj and down_proj row-split;
    * the row-split linears write fp32 partials ("partial" epilogue), which
      are all-reduced (``all_reduce``, NCCL by default) and then added to the
      residual in one rounding with the next RMSNorm fused
      (:func:`add_rms_norm`), so the rounding points are the single-GPU
      layer's; only the fp32 summation order of the split differs.  With
      ``peer`` (two :class:`parallel.PeerExchange` sites, o_proj's and
      down_proj's) the all-reduce is fused instead: each row-split linear
      stores its partial into every rank's exchange buffer over NVLink
      (:func:`draft_linear_peer`) and the add + RMSNorm sums them in rank
      order (:func:`peer_add_rms_norm`); no collective launch.

    The shard is cut from ``full``'s weights (so any world size computes the
    same layer) and packed once.  ``step`` takes the same arguments as
    :meth:`Eagle3DraftLayer.step` with the raw / working caches holding this
    rank's kv heads; :meth:`attention_partial`, :meth:`mlp_partial` and
    :meth:`finish` are its three stages between the two all-reduces."""

    def __init__(self, full: "Eagle3DraftLayer", rank: int, world: int, group=None,
                 all_reduce=None, peer=None):
        hq, hk, d, inter = full.hq, full.hk, full.d, full.inter
        if world < 1 or hq % world or (inter // world) % 64 or inter % world:
            raise ValueError("world must divide the query heads and leave the SwiGLU features "
                             "a multiple of 64 per rank")
        if world > hk and world % hk:
            raise ValueError("world must divide, or be a multiple of, the kv heads")
        self.rank, self.world, self.group = rank, world, group
        self.hq, self.d, self.eps = hq // world, d, full.eps
        self.hidden = full.w_o.shape[0]
        if world <= hk:
            self.hk = hk // world
            kv_heads = list(range(rank * self.hk, (rank + 1) * self.hk))
        else:
            self.hk = 1
            kv_heads = [rank // (world // hk)]
        self.kv_heads = kv_heads
        q0 = rank * self.hq * d
        rows_q = full.w_qkv[q0:q0 + self.hq * d]
        rows_k = torch.cat([full.w_qkv[hq * d + h * d: hq * d + (h + 1) * d] for h in kv_heads])
        rows_v = torch.cat([full.w_qkv[(hq + hk) * d + h * d: (hq + hk) * d + (h + 1) * d]
                            for h in kv_heads])
        self.w_qkv = torch.cat((rows_q, rows_k, rows_v)).contiguous()
        self.w_o = full.w_o[:, q0:q0 + self.hq * d].contiguous()
        il = inter // world
        self.inter = il
        gate = full.w_gate_up[rank * il:(rank + 1) * il]
        up = full.w_gate_up[inter + rank * il: inter + (rank + 1) * il]
        self.w_gate_up = torch.cat((gate, up)).contiguous()
        self.w_down = full.w_down[:, rank * il:(rank + 1) * il].contiguous()
        self.p_qkv = pack_linear_weight(self.w_qkv)
        self.p_o = pack_linear_weight(self.w_o)
        self.p_gate_up = pack_linear_weight(interleave_gate_up(self.w_gate_up))
        self.p_down = pack_linear_weight(self.w_down)
        self.in_norm, self.post_norm = full.in_norm, full.post_norm
        self.workspace = AttentionWorkspace(full.w_o.device)
        if all_reduce is None:
            def all_reduce(t):
                if world > 1:
                    torch.distributed.all_reduce(t, group=group)
        self.all_reduce = all_reduce
        self.peer = peer  # (o_proj site, down_proj site) or None

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for t in (self.w_qkv, self.w_o, self.w_gate_up, self.w_down))

    def attention_partial(self, x_in, *, slots, abs_positions, local_positions, raw_key,
                          raw_value, working_key, working_value, cos_sin, position_offset=0,
                          partial=None):
        """RMSNorm, this rank's q/K/V projection with the raw-cache write, RoPE,
        the draft attention over its heads and its fp32 o_proj partial."""
        n = x_in.shape[0]
        h = rms_norm(x_in, self.in_norm, self.eps)
        q, kv = qkv_projection_write_raw(h, self.p_qkv, self.hq * self.d, slots, abs_positions,
                                         raw_key, raw_value, prefetch_weight=True,
                                         packed_weight=True)
        k, v = rope_qk(q, kv, local_positions, cos_sin, self.hk, position_offset=position_offset)
        attn = draft_decode_attention(q.view(n, self.hq, self.d), k, v, working_key, working_value,
                                      slots, local_positions, self.d ** -0.5,
                                      position_offset=position_offset, workspace=self.workspace)
        return draft_linear(attn.view(n, self.hq * self.d), self.p_o, "partial", out=partial,
                            packed=True)

    def mlp_partial(self, o_sum, residual, partial=None):
        """``x = round(o_sum + residual)``, RMSNorm, this rank's gate_up +
        SwiGLU and its fp32 down_proj partial; returns ``(x, partial)``."""
        x, h2 = add_rms_norm(o_sum, residual, self.post_norm, self.eps)
        act = draft_linear(h2, self.p_gate_up, "swiglu", packed=True)
        return x, draft_linear(act, self.p_down, "partial", out=partial, packed=True)

    def finish(self, down_sum, x, out=None):
        """The layer output ``round(down_sum + x)``."""
        return add_rms_norm(down_sum, x, None, self.eps, x_out=out)[0]

    def step(self, x_in, residual, *, slots, abs_positions, local_positions, raw_key, raw_value,
             working_key, working_value, cos_sin, out=None, position_offset=0):
        """One draft step of this shard: two all-reduces of fp32 partials
        (fused into the row-split linears with ``peer``)."""
        if self.peer is not None:
            return self._step_peer(x_in, residual, slots=slots, abs_positions=abs_positions,
                                   local_positions=local_positions, raw_key=raw_key,
                                   raw_value=raw_value, working_key=working_key,
                                   working_value=working_value, cos_sin=cos_sin, out=out,
                                   position_offset=position_offset)
        po = self.attention_partial(
            x_in, slots=slots, abs_positions=abs_positions, local_positions=local_positions,
            raw_key=raw_key, raw_value=raw_value, working_key=working_key,
            working_value=working_value, cos_sin=cos_sin, position_offset=position_offset)
        self.all_reduce(po)
        x, pd = self.mlp_partial(po, residual)
        self.all_reduce(pd)
        return self.finish(pd, x, out=out)

    def attention_peer(self, x_in, *, slots, abs_positions, local_positions, raw_key, raw_value,
                       working_key, working_value, cos_sin, position_offset=0):
        """:meth:`attention_partial` with the o_proj partial stored into
        every rank's buffer of the o_proj site (fused all-reduce)."""
        n = x_in.shape[0]
        h = rms_norm(x_in, self.in_norm, self.eps)
        q, kv = qkv_projection_write_raw(h, self.p_qkv, self.hq * self.d, slots, abs_positions,
                                         raw_key, raw_value, prefetch_weight=True,
                                         packed_weight=True)
        k, v = rope_qk(q, kv, local_positions, cos_sin, self.hk, position_offset=position_offset)
        attn = draft_decode_attention(q.view(n, self.hq, self.d), k, v, working_key, working_value,
                                      slots, local_positions, self.d ** -0.5,
                                      position_offset=position_offset, workspace=self.workspace)
        draft_linear_peer(attn.view(n, self.hq * self.d), self.p_o, self.peer[0], packed=True)

    def mlp_peer(self, residual):
        """``x = round(sum of the ranks' o_proj partials + residual)`` once
        they have all arrived, RMSNorm, gate_up + SwiGLU and the down_proj
        partial into every rank's buffer of the down_proj site; returns x."""
        x, h2 = peer_add_rms_norm(self.peer[0], residual, self.post_norm, self.eps)
        act = draft_linear(h2, self.p_gate_up, "swiglu", packed=True)
        draft_linear_peer(act, self.p_down, self.peer[1], packed=True)
        return x

    def finish_peer(self, x, out=None):
        """The layer output ``round(sum of the ranks' down_proj partials + x)``."""
        return peer_add_rms_norm(self.peer[1], x, None, self.eps, x_out=out)[0]

    def _step_peer(self, x_in, residual, *, slots, abs_positions, local_positions, raw_key,
                   raw_value, working_key, working_value, cos_sin, out, position_offset):
        self.attention_peer(x_in, slots=slots, abs_positions=abs_positions,
                            local_positions=local_positions, raw_key=raw_key, raw_value=raw_value,
                            working_key=working_key, working_value=working_value, cos_sin=cos_sin,
                            position_offset=position_offset)
        return self.finish_peer(self.mlp_peer(residual), out=out)
