"""Tensor-parallel decoder over compressed weights (Qwen3 / Llama layouts).

Sharding (one process per GPU, torch.distributed / NCCL):
  * column-parallel: q_proj, k_proj, v_proj, gate_proj, up_proj and the
    vocab rows of lm_head -- rank r owns output rows [r*out/P, (r+1)*out/P),
    i.e. a contiguous run of whole chunks when the row length is a multiple
    of chunk_size, decoded with the element-range decode;
  * row-parallel: o_proj, down_proj -- rank r owns input columns
    [r*in/P, (r+1)*in/P) of every row. A TP-ready store compresses these
    tensors with a chunk_size dividing in/P_max (write_store(tp_row_chunks=...))
    so a rank's columns are whole chunks, gathered into a flat stream; for
    other chunk sizes the rank decodes the covering chunks of each row and
    slices;
  * one all-reduce (sum) after o_proj and one after down_proj per layer,
    an all-gather of the vocab shards for logits.
Heads divide across ranks (num_attention_heads and num_key_value_heads must
be multiples of P). The math mirrors transformers' Qwen3/Llama modules:
float32 RMSNorm, rotate-half RoPE with float32 cos/sin, SDPA attention.

Weights live on each rank either decoded (BF16 shards) or compressed
(`resident="compressed"`: the shard's compressed stream in HBM, decoded per
layer per forward by one batched launch).
"""
from __future__ import annotations

import dataclasses
import json
import pathlib

import numpy as np
import torch
import torch.nn.functional as F

from .. import _lib
from . import _device
from .binstore import BinaryWeightReader
from .compressed_store import CompressedLayer
from .huffman_chunked import ChunkedEncoded
from .gpu_decode_v2 import prepare_decode_tables
from .layer_decode import LayerDecoder

COL_PARALLEL = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW_PARALLEL = ("o_proj", "down_proj")


def shard_kind(key: str) -> str:
    name = key.rsplit(".", 2)[-2] if key.count(".") >= 2 else key
    if key == "lm_head.weight":
        return "col"
    if name in COL_PARALLEL:
        return "col"
    if name in ROW_PARALLEL:
        return "row"
    return "rep"


def _split(n: int, world: int, rank: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"dimension {n} does not divide across {world} ranks")
    s = n // world
    return rank * s, (rank + 1) * s


@dataclasses.dataclass
class ShardStream:
    """A rank's shard as a flat compressed stream plus how to finish it:
    decode `layer` (flat), take `rows * cols_decoded` elements from
    `elem_lo`, view them as [rows, cols_decoded] and keep columns
    [col_lo, col_lo + cols). Shards made of whole chunks need no slicing
    (elem_lo = col_lo = 0, cols = cols_decoded)."""
    layer: CompressedLayer
    rows: int
    cols_decoded: int
    col_lo: int
    cols: int
    elem_lo: int = 0

    @property
    def exact(self) -> bool:
        return self.elem_lo == 0 and self.col_lo == 0 and self.cols == self.cols_decoded and \
            int(self.layer.encoded.n_symbols) == self.rows * self.cols_decoded

    def finish(self, flat: torch.Tensor) -> torch.Tensor:
        v = flat.reshape(-1)[self.elem_lo:self.elem_lo + self.rows * self.cols_decoded]
        v = v.view(self.rows, self.cols_decoded)
        if self.col_lo or self.cols != self.cols_decoded:
            v = v[:, self.col_lo:self.col_lo + self.cols]
        return v.contiguous()


def _gather_chunks(enc, chunk_ids: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Packed bytes of the given chunks back to back, with rebased offsets."""
    offs = np.asarray(enc.chunk_offsets, dtype=np.int64)[chunk_ids]
    nbs = np.asarray(enc.chunk_nbytes, dtype=np.int64)[chunk_ids]
    packed = np.asarray(enc.packed)
    if len(chunk_ids) and np.all(np.diff(chunk_ids) == 1):
        body = packed[offs[0]:offs[-1] + nbs[-1]]
    else:
        body = np.concatenate([packed[o:o + n] for o, n in zip(offs.tolist(), nbs.tolist())]) \
            if len(chunk_ids) else np.zeros(0, np.uint8)
    new_offs = np.zeros(len(chunk_ids), dtype=np.int32)
    if len(chunk_ids) > 1:
        new_offs[1:] = np.cumsum(nbs[:-1])
    return np.concatenate([body, np.zeros(8, np.uint8)]), new_offs, nbs.astype(np.int32)


def shard_stream(layer: CompressedLayer, kind: str, world: int, rank: int) -> ShardStream:
    """The rank's shard of a 2-D compressed tensor as a flat stream
    (host-side gather; nothing is decoded here)."""
    enc = layer.encoded
    rows, cols = layer.shape
    cs = int(enc.chunk_size)
    sm = layer.sign_mantissa.reshape(-1)
    sm = sm.numpy() if isinstance(sm, torch.Tensor) else np.asarray(sm)
    n = int(enc.n_symbols)
    n_chunks = int(enc.n_chunks)
    if kind == "col":
        # output rows [r0, r1): a contiguous element range -> the chunks covering it
        r0, r1 = _split(rows, world, rank)
        e0, e1 = r0 * cols, r1 * cols
        c_lo, c_hi = e0 // cs, min(n_chunks, -(-e1 // cs))
        ids = np.arange(c_lo, c_hi, dtype=np.int64)
        sm_s = sm[c_lo * cs:min(c_hi * cs, n)]
        out_rows, dec_cols, lo, keep, elem_lo = r1 - r0, cols, 0, cols, e0 - c_lo * cs
    elif kind == "row":
        c0, c1 = _split(cols, world, rank)
        if cols % cs == 0:
            # each row's covering chunks (whole chunks when in/P is a multiple of chunk_size)
            cpr = cols // cs
            j0, j1 = c0 // cs, -(-c1 // cs)
            ids = (np.arange(rows, dtype=np.int64)[:, None] * cpr + np.arange(j0, j1)[None, :]).reshape(-1)
            sm_s = sm.reshape(rows, cols)[:, j0 * cs:j1 * cs].reshape(-1)
            out_rows, dec_cols, lo, keep, elem_lo = rows, (j1 - j0) * cs, c0 - j0 * cs, c1 - c0, 0
        else:
            # chunks straddle rows: decode the whole tensor, keep the columns
            ids = np.arange(n_chunks, dtype=np.int64)
            sm_s = sm
            out_rows, dec_cols, lo, keep, elem_lo = rows, cols, c0, c1 - c0, 0
    else:
        raise ValueError("unknown shard kind %r" % kind)
    packed, offs, nbs = _gather_chunks(enc, ids)
    n_dec = int(sm_s.shape[0])
    enc_s = ChunkedEncoded(packed=packed, chunk_offsets=offs, chunk_nbytes=nbs, sym_lut=enc.sym_lut,
                           len_lut=enc.len_lut, max_bits=enc.max_bits, chunk_size=cs, n_symbols=n_dec,
                           shape=(n_dec,))
    return ShardStream(CompressedLayer(sign_mantissa=torch.from_numpy(np.ascontiguousarray(sm_s)), encoded=enc_s,
                                       shape=(n_dec,)), out_rows, dec_cols, lo, keep, elem_lo)


def _mark(stream) -> torch.cuda.Event:
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream)
    return ev


def _union(iv: list[tuple[float, float]]) -> list[tuple[float, float]]:
    out: list[list[float]] = []
    for a, b in sorted(iv):
        if out and a <= out[-1][1]:
            out[-1][1] = max(out[-1][1], b)
        else:
            out.append([a, b])
    return [(a, b) for a, b in out]


def _measure(iv: list[tuple[float, float]]) -> float:
    return sum(b - a for a, b in iv)


def _intersect(x: list[tuple[float, float]], y: list[tuple[float, float]]) -> float:
    i = j = 0
    tot = 0.0
    while i < len(x) and j < len(y):
        a, b = max(x[i][0], y[j][0]), min(x[i][1], y[j][1])
        if b > a:
            tot += b - a
        if x[i][1] < y[j][1]:
            i += 1
        else:
            j += 1
    return tot


def timeline_summary(timeline: list, base: torch.cuda.Event) -> dict:
    """Busy time of each kind of work (decode launches, per-layer compute,
    host->device layer copies) from CUDA events, and how much of it ran
    concurrently: `decode_overlapped_ms` is decode time during which the
    compute stream was also busy. Call after synchronising."""
    iv: dict[str, list] = {}
    rows = []
    for kind, layer, a, b in timeline:
        t0, t1 = base.elapsed_time(a), base.elapsed_time(b)
        iv.setdefault(kind, []).append((t0, t1))
        rows.append((kind, layer, round(t0, 4), round(t1, 4)))
    u = {k: _union(v) for k, v in iv.items()}
    span = (min(a for v in u.values() for a, _ in v), max(b for v in u.values() for _, b in v)) if u else (0, 0)
    out = {"span_ms": round(span[1] - span[0], 4)}
    for k, v in u.items():
        out[k + "_busy_ms"] = round(_measure(v), 4)
    if "decode" in u and "compute" in u:
        out["decode_overlapped_ms"] = round(_intersect(u["decode"], u["compute"]), 4)
    if "upload" in u:
        busy = _union(u.get("decode", []) + u.get("compute", []))
        out["upload_overlapped_ms"] = round(_intersect(u["upload"], busy), 4)
    out["events"] = rows
    return out


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    h = x.to(torch.float32)
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(dt)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class KVCache:
    """Static per-rank cache: [layers][2] tensors of [1, kv_heads_local, max_len, head_dim]."""

    def __init__(self, n_layers, kv_heads, head_dim, max_len, device, dtype=torch.bfloat16):
        self.k = [torch.zeros(1, kv_heads, max_len, head_dim, device=device, dtype=dtype) for _ in range(n_layers)]
        self.v = [torch.zeros(1, kv_heads, max_len, head_dim, device=device, dtype=dtype) for _ in range(n_layers)]
        self.max_len = max_len
        self.length = 0


class _StepState:
    """Static buffers of the graphed single-token step."""

    def __init__(self, dec: "TPDecoder", max_len: int):
        dev = dec.device
        self.max_len = max_len
        self.cache = KVCache(dec.n_layers, dec.nkv, dec.hd, max_len, dev)
        self.ids = torch.zeros(1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.step = torch.zeros(1, dtype=torch.long, device=dev)
        self.tokens = torch.zeros(max_len, dtype=torch.long, device=dev)
        self.arange = torch.arange(max_len, device=dev).view(1, max_len)
        self.mask = torch.zeros(1, max_len, dtype=torch.bool, device=dev)  # [query, key]
        self.graph = None
        self.prefill: dict = {}   # prompt length -> (graph, static prompt buffer)
        self.pool = torch.cuda.graph_pool_handle()


class TPDecoder:
    """One rank of a tensor-parallel decoder. `group` is a torch.distributed
    process group (None for a single rank)."""

    def __init__(self, hf_cfg, weights: dict, world: int = 1, rank: int = 0, group=None, device="cuda",
                 fused: bool = True):
        self.cfg = hf_cfg
        self.world, self.rank, self.group = world, rank, group
        self.device = torch.device(device)
        # single-token forwards use the fused layer kernels (csrc/tp_ops.cu); the torch
        # layer math remains for prompts, and for CPU ranks (host-logic tests)
        self.fused = bool(fused) and self.device.type == "cuda"
        self.H = hf_cfg.hidden_size
        self.hd = getattr(hf_cfg, "head_dim", None) or self.H // hf_cfg.num_attention_heads
        self.nh = hf_cfg.num_attention_heads // world
        self.nkv = hf_cfg.num_key_value_heads // world
        if hf_cfg.num_attention_heads % world or hf_cfg.num_key_value_heads % world:
            raise ValueError("attention heads do not divide across %d ranks" % world)
        self.eps = hf_cfg.rms_norm_eps
        self.n_layers = hf_cfg.num_hidden_layers
        self.qk_norm = "model.layers.0.self_attn.q_norm.weight" in weights
        self.vocab = hf_cfg.vocab_size
        self.w = weights  # key -> tensor (shard) or a callable returning it
        self.timeline = None  # a list to record (kind, layer, start event, end event) into
        self._graph_state = None
        self.allreducer = None  # one-shot NVLink all-reduce (use_oneshot_allreduce); else NCCL
        rp = getattr(hf_cfg, "rope_parameters", None) or {}
        theta = rp.get("rope_theta", getattr(hf_cfg, "rope_theta", 10000.0))
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, self.hd, 2, dtype=torch.int64).to(
            device=self.device, dtype=torch.float) / self.hd))
        if self.fused:
            self._join_resident()

    # q/k/v (and gate/up) consume the same input: stored back to back they are one projection
    JOINS = (("self_attn.qkv_proj.weight", ("self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                            "self_attn.v_proj.weight")),
             ("mlp.gate_up_proj.weight", ("mlp.gate_proj.weight", "mlp.up_proj.weight")))

    def _join_resident(self) -> None:
        """Resident BF16 shards of q/k/v and of gate/up are moved into one
        buffer each; the separate names stay as views of it."""
        for i in range(self.n_layers):
            p = "model.layers.%d." % i
            for joined, names in self.JOINS:
                parts = [self.w.get(p + n) for n in names]
                if any(t is None or callable(t) or t.dim() != 2 for t in parts):
                    continue
                if len({t.shape[1] for t in parts}) != 1:
                    continue
                buf = torch.cat(parts, 0)
                r = 0
                for n, t in zip(names, parts):
                    self.w[p + n] = buf[r:r + t.shape[0]]
                    r += t.shape[0]
                self.w[p + joined] = buf

    @staticmethod
    def _adjacent(parts: list) -> torch.Tensor | None:
        """One [sum of rows, cols] view over 2-D tensors stored back to back
        in one buffer, or None."""
        first = parts[0]
        cols = first.shape[1]
        end = first.data_ptr()
        for t in parts:
            if t.dim() != 2 or t.shape[1] != cols or not t.is_contiguous() or t.dtype != first.dtype \
                    or t.data_ptr() != end:
                return None
            end += t.numel() * t.element_size()
        rows = sum(t.shape[0] for t in parts)
        return torch.as_strided(first, (rows, cols), (cols, 1))

    def _joined(self, W: dict, joined: str, names: tuple) -> torch.Tensor:
        t = W.get(joined)
        if t is not None:
            return t
        parts = [W[n] for n in names]
        t = self._adjacent(parts)
        return t if t is not None else torch.cat(parts, 0)

    # -- weights -----------------------------------------------------------
    def weight(self, key: str) -> torch.Tensor:
        w = self.w[key]
        return w() if callable(w) else w

    # -- collectives ----------------------------------------------------------
    def use_oneshot_allreduce(self, max_floats: int = 1 << 16) -> None:
        """Collective (every rank calls it): the row-parallel sums of up to
        max_floats floats go through the one-shot NVLink all-reduce
        (runtime/allreduce.py, csrc/allreduce.cu) instead of NCCL; larger
        ones (long prompts) stay on NCCL. A CPU or single-rank decoder keeps
        what it has."""
        if self.world < 2 or self.device.type != "cuda" or self.allreducer is not None:
            return
        from .allreduce import OneShotAllReduce
        try:
            self.allreducer = OneShotAllReduce(self.group, self.device, max_floats)
        except ValueError:  # ranks that share a GPU keep NCCL (every rank sees the same answer)
            self.allreducer = None

    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            torch.distributed.all_reduce(x, group=self.group)
        return x

    # projections at least this many output rows wide run on this package's kernels in the
    # fused mode (measured on B200: at or above cuBLAS from here on up, below it for narrower ones)
    OWN_KERNEL_MIN_ROWS = 16384

    def _proj(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x @ w.T for a column-parallel projection or the head. In the fused
        mode a wide projection (>= OWN_KERNEL_MIN_ROWS output rows: gate/up,
        the vocabulary head) runs on csrc/gemv.cu for up to 8 tokens and on
        the tcgen05 tensor-core GEMM (csrc/gemm_tc.cu) for 9..64 tokens; both
        keep fp32 sums and round once. Everything else, and the unfused mode,
        is F.linear, the call transformers makes."""
        if self.fused and w.shape[0] >= self.OWN_KERNEL_MIN_ROWS and w.dim() == 2 and w.stride(-1) == 1 \
                and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16:
            from . import tp_ops
            x2 = x.reshape(-1, x.shape[-1])
            T, K = x2.shape
            if x2.stride(-1) == 1 and K % 8 == 0 and w.stride(0) % 8 == 0 and x2.stride(0) % 8 == 0 \
                    and x2.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0:
                if T <= 8:
                    return tp_ops.gemv(x2, w).reshape(*x.shape[:-1], w.shape[0])
                if T <= 64 and K % 64 == 0:
                    return tp_ops.gemm_tc(x2, w).reshape(*x.shape[:-1], w.shape[0])
        return F.linear(x, w)

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x @ w.T for a row-parallel projection (o_proj, down_proj), summed
        over the ranks. On one rank it is F.linear, the call transformers
        makes. On several ranks each rank's partial product stays in fp32,
        the all-reduce sums fp32, and the sum is rounded to BF16 once: a
        single GEMM's rounding, rather than a rounding of every rank's partial
        plus one per summation in BF16."""
        if self.world == 1:
            return F.linear(x, w)
        x2 = x.reshape(-1, x.shape[-1])
        if x2.device.type == "cuda":
            y = torch.mm(x2, w.t(), out_dtype=torch.float32)
        else:
            y = x2.float() @ w.float().t()
        t0 = _mark(torch.cuda.current_stream(self.device)) \
            if self.timeline is not None and self.device.type == "cuda" else None
        if self.allreducer is not None and y.numel() <= self.allreducer.max_floats:
            self.allreducer(y)
        else:
            torch.distributed.all_reduce(y, group=self.group)
        if t0 is not None:
            self.timeline.append(("allreduce", -1, t0, _mark(torch.cuda.current_stream(self.device))))
        return y.to(x.dtype).reshape(*x.shape[:-1], w.shape[0])

    def _all_gather_last(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.world)]
        torch.distributed.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    # -- forward -------------------------------------------------------------
    def _rope(self, positions: torch.Tensor, dtype):
        freqs = positions[:, None].float() * self.inv_freq[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(dtype), emb.sin().to(dtype)

    def layer_weights(self, i: int) -> dict:
        """Hook point: the compressed-resident subclass decodes here."""
        p = "model.layers.%d." % i
        names = ["input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                 "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                 "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]
        if self.qk_norm:
            names += ["self_attn.q_norm.weight", "self_attn.k_norm.weight"]
        return {n: self.weight(p + n) for n in names}

    def _layer(self, i: int, x: torch.Tensor, cos, sin, cache: KVCache | None, start: int,
               static=None) -> torch.Tensor:
        W = self.layer_weights(i)
        if self.timeline is None:
            return self._layer_math(i, W, x, cos, sin, cache, start, static)
        t0 = _mark(torch.cuda.current_stream(self.device))
        x = self._layer_math(i, W, x, cos, sin, cache, start, static)
        self.timeline.append(("compute", i, t0, _mark(torch.cuda.current_stream(self.device))))
        return x

    def _layer_math(self, i: int, W: dict, x: torch.Tensor, cos, sin, cache: KVCache | None,
                    start: int, static=None) -> torch.Tensor:
        T = x.shape[0]
        h = _rms_norm(x, W["input_layernorm.weight"], self.eps)
        q = F.linear(h, W["self_attn.q_proj.weight"]).view(T, self.nh, self.hd)
        k = F.linear(h, W["self_attn.k_proj.weight"]).view(T, self.nkv, self.hd)
        v = F.linear(h, W["self_attn.v_proj.weight"]).view(T, self.nkv, self.hd)
        if self.qk_norm:
            q = _rms_norm(q, W["self_attn.q_norm.weight"], self.eps)
            k = _rms_norm(k, W["self_attn.k_norm.weight"], self.eps)
        q, k, v = q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None]
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        if static is not None:
            # single-token step with static shapes (CUDA-graph safe): the position is a
            # device tensor, attention runs over the whole cache with a length mask
            cache.k[i].index_copy_(2, static.pos, k)
            cache.v[i].index_copy_(2, static.pos, v)
            k, v = cache.k[i], cache.v[i]
        elif cache is not None:
            cache.k[i][:, :, start:start + T] = k
            cache.v[i][:, :, start:start + T] = v
            k = cache.k[i][:, :, :start + T]
            v = cache.v[i][:, :, :start + T]
        L = k.shape[2]
        if static is not None:
            mask = static.mask
        elif T == 1:
            mask = None
        else:
            qpos = torch.arange(start, start + T, device=x.device)[:, None]
            mask = torch.arange(L, device=x.device)[None, :] <= qpos
        a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=self.hd ** -0.5,
                                           enable_gqa=self.nh != self.nkv)
        a = a[0].transpose(0, 1).reshape(T, self.nh * self.hd)
        x = x + self._row_parallel(a, W["self_attn.o_proj.weight"])
        h = _rms_norm(x, W["post_attention_layernorm.weight"], self.eps)
        m = F.silu(self._proj(h, W["mlp.gate_proj.weight"])) * self._proj(h, W["mlp.up_proj.weight"])
        return x + self._row_parallel(m, W["mlp.down_proj.weight"])

    def _layer_fused(self, i: int, W: dict, x: torch.Tensor, delta, cache: KVCache,
                     pos: torch.Tensor) -> torch.Tensor:
        """One layer for one token with the fused kernels. x [1, H] is the
        residual stream, updated in place with the previous layer's pending
        MLP output `delta`; returns this layer's (all-reduced) MLP output,
        which the next norm adds. Same math as _layer_math."""
        from . import tp_ops
        h = tp_ops.add_rmsnorm(x, delta, W["input_layernorm.weight"], self.eps)
        qkv = F.linear(h, self._joined(W, *self.JOINS[0]))
        q = torch.empty(self.nh, 1, self.hd, dtype=x.dtype, device=x.device)
        qn = W.get("self_attn.q_norm.weight") if self.qk_norm else None
        kn = W.get("self_attn.k_norm.weight") if self.qk_norm else None
        tp_ops.qk_rope_cache(qkv, 1, self.nh, self.nkv, self.hd, qn, kn, self.eps, self.inv_freq, pos, q,
                             cache.k[i], cache.v[i])
        a = tp_ops.decode_attention(q, cache.k[i], cache.v[i], self.nh, self.nkv, self.hd, pos, self.hd ** -0.5)
        o = self._row_parallel(a[None], W["self_attn.o_proj.weight"])
        h = tp_ops.add_rmsnorm(x, o, W["post_attention_layernorm.weight"], self.eps)
        m = tp_ops.silu_mul(self._proj(h, self._joined(W, *self.JOINS[1])))
        return self._row_parallel(m, W["mlp.down_proj.weight"])

    def _layers_fused(self, x: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        """Every layer for one token, then the final norm; returns the
        normalised hidden state [1, H]."""
        from . import tp_ops
        delta = None
        for i in range(self.n_layers):
            W = self.layer_weights(i)
            t0 = _mark(torch.cuda.current_stream(self.device)) if self.timeline is not None else None
            delta = self._layer_fused(i, W, x, delta, cache, pos)
            if t0 is not None:
                self.timeline.append(("compute", i, t0, _mark(torch.cuda.current_stream(self.device))))
        return tp_ops.add_rmsnorm(x, delta, self.weight("model.norm.weight"), self.eps)

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        e = self.w["model.embed_tokens.weight"]
        if callable(e):
            return e(ids)
        return F.embedding(ids, e)

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, cache: KVCache | None = None) -> torch.Tensor:
        """Logits [T, vocab] for the T tokens of `input_ids` (batch 1),
        appended to `cache` when given."""
        ids = input_ids.reshape(-1).to(self.device)
        start = cache.length if cache is not None else 0
        T = ids.shape[0]
        self.begin_forward()
        x = self.embed(ids)
        if self.fused and T == 1 and cache is not None and start < cache.max_len:
            pos_t = torch.full((1,), start, dtype=torch.int64, device=self.device)
            h = self._layers_fused(x.contiguous(), cache, pos_t)
            cache.length = start + 1
            return self._all_gather_last(self.head_logits(h))
        pos = torch.arange(start, start + T, device=self.device)
        cos, sin = self._rope(pos, x.dtype)
        for i in range(self.n_layers):
            x = self._layer(i, x, cos, sin, cache, start)
        if cache is not None:
            cache.length = start + T
        x = _rms_norm(x, self.weight("model.norm.weight"), self.eps)
        return self._all_gather_last(self.head_logits(x))

    def begin_forward(self) -> None:
        """Hook run at the start of every forward (stream forks)."""

    def _static_step(self, st: "_StepState") -> None:
        """One greedy single-token step on static buffers: embeds st.ids at
        position st.pos, runs every layer, picks the argmax token, records it
        at st.tokens[st.step] and advances ids/pos/step -- all on the
        device, so the step can be captured and replayed as a CUDA graph."""
        self.begin_forward()
        x = F.embedding(st.ids, self.weight("model.embed_tokens.weight"))
        if self.fused:
            x = self._layers_fused(x, st.cache, st.pos)
        else:
            cos, sin = self._rope(st.pos, x.dtype)
            torch.le(st.arange, st.pos, out=st.mask)
            for i in range(self.n_layers):
                x = self._layer(i, x, cos, sin, st.cache, 0, static=st)
            x = _rms_norm(x, self.weight("model.norm.weight"), self.eps)
        logits = self._all_gather_last(self.head_logits(x))
        nxt = logits[-1].argmax(-1, keepdim=True)
        st.tokens.index_copy_(0, st.step, nxt)
        st.ids.copy_(nxt)
        st.pos.add_(1)
        st.step.add_(1)

    @torch.no_grad()
    def generate_greedy_graphed(self, input_ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy decoding from CUDA graphs: the prompt pass is captured once
        per prompt length (static shapes: positions 0..P-1, causal mask) and
        the single-token step once (decode launches, projections,
        all-reduces, argmax and the position update); both are replayed.
        Each graph is captured after one eager run of the same work (cuBLAS,
        NCCL and allocator state). The embedding must be on the device."""
        if callable(self.w.get("model.embed_tokens.weight")) or getattr(self, "mode", None) == "streamed":
            raise ValueError("graphed generation needs device-resident weights and embedding "
                             "(resident='decoded' or 'compressed')")
        ids = input_ids.reshape(1, -1).to(self.device)
        P = ids.shape[1]
        if max_new_tokens < 1:
            return ids
        st = self._graph_state
        if st is None or st.max_len < P + max_new_tokens:
            self.release_graphs()
            # 64 positions of room past the generation for replay_steps to continue it
            st = _StepState(self, max(128, P + max_new_tokens + 64))
            self._graph_state = st
        pre = st.prefill.get(P)
        if pre is None:
            buf = ids.reshape(-1).clone()
            self._prefill_into(st, buf)  # eager run of the same work
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=st.pool):
                self._prefill_into(st, buf)
            pre = (g, buf)
            st.prefill[P] = pre
        g, buf = pre
        buf.copy_(ids.reshape(-1))
        g.replay()
        first = st.ids.clone()
        if max_new_tokens == 1:
            return torch.cat([ids, first.reshape(1, 1)], 1)
        st.pos.fill_(P)
        st.step.zero_()
        todo = max_new_tokens - 1
        if st.graph is None:
            # one real step eagerly on a side stream, then capture
            cur = torch.cuda.current_stream(self.device)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                self._static_step(st)
            cur.wait_stream(side)
            torch.cuda.synchronize(self.device)
            todo -= 1
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=st.pool):
                self._static_step(st)
            st.graph = g
        for _ in range(todo):
            st.graph.replay()
        out = torch.cat([ids, first.reshape(1, 1), st.tokens[:max_new_tokens - 1].reshape(1, -1)], 1)
        _device.check_status(self.device)  # a corrupt stream in any replayed decode raises here
        return out

    def _prefill_into(self, st: "_StepState", prompt: torch.Tensor) -> None:
        """The prompt pass from an empty cache, leaving its greedy token in
        st.ids (static shapes for a fixed prompt length)."""
        st.cache.length = 0
        logits = self.forward(prompt, st.cache)
        st.ids.copy_(logits[-1:].argmax(-1).reshape(1))

    @torch.no_grad()
    def replay_steps(self, n: int) -> int:
        """Replays the captured single-token step up to n more times,
        continuing the last graphed generation (for timing the step alone);
        returns how many ran (bounded by the static cache length)."""
        st = self._graph_state
        if st is None or st.graph is None:
            raise RuntimeError("no captured step: call generate_greedy_graphed first")
        used = int(st.pos.item())
        k = max(0, min(n, st.max_len - used, st.max_len - int(st.step.item())))
        for _ in range(k):
            st.graph.replay()
        return k

    def release_graphs(self) -> None:
        """Drops the captured step (release before destroying the process group)."""
        self._graph_state = None

    def close(self) -> None:
        """Collective when the one-shot all-reduce is in use."""
        self.release_graphs()
        if self.allreducer is not None:
            self.allreducer.close()
            self.allreducer = None

    def head_logits(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's vocab shard of the logits."""
        head = self.w.get("lm_head.weight", None)
        return self._proj(x, self.weight("lm_head.weight") if head is not None else self.full_embed_shard())

    def full_embed_shard(self) -> torch.Tensor:
        """Tied head: this rank's vocab rows of the (replicated) embedding."""
        e = self.weight("model.embed_tokens.weight")
        v0, v1 = _split(self.vocab, self.world, self.rank)
        return e[v0:v1]

    @torch.no_grad()
    def generate_greedy(self, input_ids: torch.Tensor, max_new_tokens: int, max_len: int | None = None):
        ids = input_ids.reshape(1, -1)
        max_len = max_len or ids.shape[1] + max_new_tokens
        cache = KVCache(self.n_layers, self.nkv, self.hd, max_len, self.device)
        seq = ids.to(self.device)
        step = seq
        for _ in range(max_new_tokens):
            logits = self.forward(step, cache)
            nxt = logits[-1:].argmax(-1).reshape(1, 1)
            seq = torch.cat([seq, nxt], 1)
            step = nxt
        _device.check_status(self.device)  # a corrupt stream in any decode of the run raises here
        return seq

    @torch.no_grad()
    def generate_speculative(self, input_ids: torch.Tensor, max_new_tokens: int, draft: "TPDecoder", k: int = 4,
                             temperature: float = 0.0, generator: torch.Generator | None = None,
                             stats: dict | None = None) -> torch.Tensor:
        """Draft/target speculation with a KV cache on both models (the
        reference's loop, streaming_engine.py:2488-2575; acceptance by
        verify.py:53-103 through speculative_sample_step). `draft` is another
        decoder on the same ranks with the same vocabulary (the benchmark
        pairs the Qwen3-14B shape with a Qwen3-0.6B-shaped draft).

        Each sweep: the draft proposes k tokens one at a time (its
        single-token steps); the target scores the pending token and the k
        proposals in ONE (k+1)-token forward at the end of its cache; an
        accepted prefix plus one correction or bonus token is committed, and
        both caches are cut back to the committed tokens. The reference
        instead re-runs the whole sequence through the target every sweep.
        At temperature <= 0 the accepted tokens are the target's argmax, so
        the output is greedy decoding's, up to BF16 rounding differences
        between the (k+1)-token and the one-token forward. Every rank takes
        the same decisions: the logits are all-gathered, and a generator
        must be seeded alike on every rank."""
        from .verify import sample_categorical, speculative_sample_step, temperature_probs
        if draft.vocab != self.vocab:
            raise ValueError("the draft's vocabulary (%d) does not match the target's (%d)"
                             % (draft.vocab, self.vocab))
        if k < 1:
            raise ValueError("k must be >= 1")
        ids = input_ids.reshape(1, -1).to(self.device)
        P = ids.shape[1]
        if max_new_tokens < 1:
            return ids
        max_len = P + max_new_tokens + k + 2
        tc = KVCache(self.n_layers, self.nkv, self.hd, max_len, self.device)
        dc = KVCache(draft.n_layers, draft.nkv, draft.hd, max_len, draft.device)
        # the first token comes from the target's prompt pass, as in greedy decoding;
        # the target cache then holds every committed token but the last (pending) one
        first = temperature_probs(self.forward(ids, tc)[-1], temperature)
        committed = ids[0].tolist() + [sample_categorical(first, generator) if temperature > 0
                                       else int(first.argmax())]
        sweeps = accepted_total = 0
        while len(committed) - P < max_new_tokens:
            # draft: catch up on committed tokens it has not seen, then propose k
            todo = committed[dc.length:]
            lg = draft.forward(torch.tensor([todo], device=draft.device), dc)[-1]
            d_tokens, d_probs = [], []
            for j in range(k):
                q = temperature_probs(lg, temperature)
                t = sample_categorical(q, generator) if temperature > 0 else int(q.argmax())
                d_tokens.append(t)
                d_probs.append(q)
                if j + 1 < k:
                    lg = draft.forward(torch.tensor([[t]], device=draft.device), dc)[-1]
            # target: the pending token and the k proposals in one forward
            base = len(committed) - 1
            tl = self.forward(torch.tensor([[committed[-1]] + d_tokens], device=self.device), tc)
            t_probs = [temperature_probs(tl[i], temperature) for i in range(k)]
            bonus = temperature_probs(tl[k], temperature)
            if temperature > 0:
                new, n_draft = speculative_sample_step(d_probs, t_probs, d_tokens, bonus, generator)
            else:
                # one-hot distributions: accept while the proposal is the target's argmax
                new, n_draft = [], k
                for i, t in enumerate(d_tokens):
                    best = int(t_probs[i].argmax())
                    new.append(best)
                    if best != t:
                        n_draft = i
                        break
                else:
                    new.append(int(bonus.argmax()))
            committed += new
            tc.length = base + 1 + n_draft  # cut the rejected proposals (and their KV entries)
            dc.length = min(dc.length, base + 1 + n_draft)
            sweeps += 1
            accepted_total += n_draft
        if stats is not None:
            stats.update(sweeps=sweeps, accepted_from_draft=accepted_total, k=k)
        _device.check_status(self.device)
        _device.check_status(draft.device)
        return torch.tensor([committed[:P + max_new_tokens]], device=self.device)


_ALIGN = 256


class HostArena:
    """One page-locked host allocation of exactly `nbytes` (an anonymous
    mapping registered with the CUDA driver), so that uploads from it are
    asynchronous DMA copies; torch's pinned allocator would round every
    block up to a power of two."""

    def __init__(self, nbytes: int):
        import mmap
        self.nbytes = max(int(nbytes), 4096)
        self._map = mmap.mmap(-1, self.nbytes)
        self.array = np.frombuffer(self._map, dtype=np.uint8)
        err = torch._C._cudart.cudaHostRegister(self.array.ctypes.data, self.nbytes, 0)
        if int(err) != 0:
            raise RuntimeError("cudaHostRegister of %d bytes failed (%s)" % (self.nbytes, err))
        self.tensor = torch.from_numpy(self.array)

    def close(self) -> None:
        if self._map is not None:
            torch._C._cudart.cudaHostUnregister(self.array.ctypes.data)
            self.tensor = None
            self.array = None
            self._map = None  # released with the last view


@dataclasses.dataclass
class _Seg:
    """Where one shard's stream sits inside its layer's byte image."""
    key: str
    ss: ShardStream
    tables: object
    packed_off: int
    packed_n: int
    packed_cap: int
    offs_off: int
    nbs_off: int
    n_chunks: int
    sm_off: int


def _up(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


def _layer_layout(streams: list[tuple[str, ShardStream]], tables: dict) -> tuple[list[_Seg], int]:
    segs, pos = [], 0
    for key, ss in streams:
        enc = ss.layer.encoded
        pn = int(np.asarray(enc.packed).shape[0])
        cap = max(16, (pn + 15) // 16 * 16)
        nc = int(enc.n_chunks)
        seg = _Seg(key, ss, tables[key], pos, pn, cap, 0, 0, nc, 0)
        pos = _up(pos + cap)
        seg.offs_off = pos
        pos = _up(pos + 4 * max(nc, 1))
        seg.nbs_off = pos
        pos = _up(pos + 4 * max(nc, 1))
        seg.sm_off = pos
        pos = _up(pos + int(ss.layer.sign_mantissa.numel()))
        segs.append(seg)
    return segs, pos


def _fill_image(dst: np.ndarray, segs: list[_Seg]) -> None:
    for g in segs:
        enc = g.ss.layer.encoded
        dst[g.packed_off:g.packed_off + g.packed_n] = np.asarray(enc.packed)
        dst[g.packed_off + g.packed_n:g.packed_off + g.packed_cap] = 0
        dst[g.offs_off:g.offs_off + 4 * g.n_chunks] = np.asarray(enc.chunk_offsets, dtype=np.int32).view(np.uint8)
        dst[g.nbs_off:g.nbs_off + 4 * g.n_chunks] = np.asarray(enc.chunk_nbytes, dtype=np.int32).view(np.uint8)
        sm = g.ss.layer.sign_mantissa.reshape(-1).numpy()
        dst[g.sm_off:g.sm_off + sm.shape[0]] = sm


def plan_resident_layers(layer_bytes: list[int], vram_budget_bytes: int, fixed_bytes: int) -> list[int]:
    """Which layer images a streamed rank keeps in HBM under a per-rank VRAM
    budget: the residency planner (vram_planner.plan_tiers) run on this
    rank's shard images, with the rank's fixed working set (slot ring,
    decode outputs, head, tables, activations) as headroom. Raises if the
    budget cannot hold the working set."""
    from .vram_planner import TensorInfo, plan_tiers
    infos = [TensorInfo(key="layer.%d" % i, orig_bytes=int(n), comp_bytes=int(n), is_layer_weight=True)
             for i, n in enumerate(layer_bytes)]
    plan = plan_tiers(infos, vram_budget_bytes / 1e9, 0.0, vram_headroom_bytes=int(fixed_bytes))
    if not plan.feasible:
        raise ValueError("per-rank VRAM budget %.2f GB is below this rank's streaming working set %.2f GB"
                         % (vram_budget_bytes / 1e9, fixed_bytes / 1e9))
    return sorted(int(k.split(".")[1]) for k in plan.vram_keys)


class CompressedTPDecoder(TPDecoder):
    """TP decoder whose projection shards stay compressed; each layer's
    shards are decoded by one batched launch per forward, straight into
    the [rows, cols] weights (the element range skips a column shard's
    partial leading chunk).

    Each layer's shards form one byte image: per tensor the packed stream
    (16-byte padded), int32 chunk offsets and byte counts, and the
    sign/mantissa bytes, each 256-byte aligned.
      * mode="compressed": every image resident in HBM (uploaded once).
      * mode="streamed": images in page-locked host memory; `slots` device
        buffers hold the next layers, filled by one copy per layer on a
        copy stream that runs ahead of the compute stream (layer i+slots
        uploads into layer i's buffer as soon as its decode has run), so
        the PCIe transfer overlaps decode and projection. With a per-rank
        `vram_budget_gb`, the planner keeps as many layer images resident in
        HBM as the budget allows beside that working set; only the rest
        stream.
    The head (vocab rows of lm_head, or of a tied embedding) stays compressed
    in HBM and is decoded `head_block_rows` rows at a time into one reused
    buffer, so it never exists decoded in full. With `overlap`, layer i+1 is
    decoded on a side stream while layer i's projections run; `decode_sms`
    (> 0) caps that decode's CTAs (one per SM) so that the projections get
    the remaining SMs instead of queueing behind it."""

    def __init__(self, hf_cfg, weights: dict, streams: dict, world=1, rank=0, group=None, device="cuda",
                 mode: str = "compressed", slots: int = 3, head_block_rows: int = 16384, overlap: bool = False,
                 fused: bool = True, vram_budget_gb: float | None = None, max_context: int = 4096,
                 decode_sms: int | None = None):
        super().__init__(hf_cfg, weights, world, rank, group, device, fused=fused)
        if mode not in ("compressed", "streamed"):
            raise ValueError("mode must be 'compressed' or 'streamed'")
        self.dev = _device.cuda_device(device)
        self.mode = mode
        self.decoder = LayerDecoder(self.dev)
        self.tables = {k: prepare_decode_tables(ss.layer.encoded, self.dev) for k, ss in streams.items()}
        self.layer_keys = [[k for k, v in self.w.items() if v is not None and k.startswith("model.layers.%d." % i)]
                           for i in range(self.n_layers)]
        self.segs, sizes = [], []
        for i in range(self.n_layers):
            pre = "model.layers.%d." % i
            segs, nb = _layer_layout([(k, ss) for k, ss in streams.items() if k.startswith(pre)], self.tables)
            self.segs.append(segs)
            sizes.append(nb)
        head_key = "lm_head.weight" if "lm_head.weight" in streams else None
        self.head = None
        if head_key is not None:
            hsegs, hn = _layer_layout([(head_key, streams[head_key])], self.tables)
            img = np.zeros(hn, dtype=np.uint8)
            _fill_image(img, hsegs)
            self.head = (hsegs[0], torch.from_numpy(img).to(self.dev))
            self.head_block_rows = max(1, int(head_block_rows))
        self._desc_cache: dict = {}
        self.overlap = bool(overlap)
        self._dec_stream = torch.cuda.Stream(self.dev) if self.overlap else None
        # with overlap: SMs the side-stream layer decode may hold (0 = all); the
        # rest stay free for the current layer's projections. The default, 78 %
        # of the SMs, is the best of a sweep of the 14B shape's graphed step at
        # TP=1 on B200 (116 of 148 SMs: 18.1 -> 16.6 ms; 92 SMs: 20.7 ms)
        if decode_sms is None:
            decode_sms = round(0.78 * torch.cuda.get_device_properties(self.dev).multi_processor_count)
        self.decode_sms = int(decode_sms) if self.overlap else 0
        self._ahead: dict = {}
        # decoded weights land in preallocated output sets (two when the decode of layer
        # i+1 overlaps layer i's projections), so descriptors are built once per
        # (layer, image, set) and nothing is allocated per layer
        per_layer = [self._out_layout(segs) for segs in self.segs]
        set_elems = max([n for _, n in per_layer] + [1])
        self._out_sets = [torch.empty(set_elems, dtype=torch.bfloat16, device=self.dev)
                          for _ in range(2 if self.overlap else 1)]
        self._out_offs = [o for o, _ in per_layer]
        self._set_free = [None] * len(self._out_sets)
        if self.head is not None:
            g = self.head[0]
            rows = min(self.head_block_rows, g.ss.rows)
            self._head_buf = torch.empty(rows * g.ss.cols_decoded, dtype=torch.bfloat16, device=self.dev)
        resident = set(range(self.n_layers))
        self.budget_plan = None
        if mode == "streamed":
            resident = set()
            if vram_budget_gb is not None:
                n_slots = max(1, slots)
                fixed = (n_slots * _up(max(max(sizes), 16)) + sum(t.numel() * 2 for t in self._out_sets)
                         + (self.head[1].numel() + self._head_buf.numel() * 2 if self.head is not None else 0)
                         + sum(t.block.numel() + t.sym_lut.numel() * 4 + t.len_lut.numel()
                               for t in self.tables.values())
                         + 2 * self.n_layers * self.nkv * self.hd * 2 * max_context
                         # device-resident tensors outside the layers (a tied embedding, norms)
                         + sum(t.numel() * t.element_size() for k, t in self.w.items()
                               if isinstance(t, torch.Tensor) and t.device.type == "cuda"
                               and not k.startswith("model.layers."))
                         + (256 << 20))  # activations of a prompt pass, logits, allocator slack
                resident = set(plan_resident_layers(sizes, int(vram_budget_gb * 1e9), fixed))
                self.budget_plan = {"vram_budget_gb": vram_budget_gb, "fixed_bytes": int(fixed),
                                    "resident_layers": len(resident), "streamed_layers": self.n_layers - len(resident)}
        self.images = {}
        for i in sorted(resident):
            img = np.zeros(max(sizes[i], 16), dtype=np.uint8)
            _fill_image(img, self.segs[i])
            self.images[i] = torch.from_numpy(img).to(self.dev)
        self.streamed = [i for i in range(self.n_layers) if i not in resident]
        self._stream_pos = {layer: j for j, layer in enumerate(self.streamed)}
        self.h2d_bytes = 0
        self.host = {}
        if self.streamed:
            ssz = [_up(max(sizes[i], 16)) for i in self.streamed]
            offs = np.concatenate([[0], np.cumsum(ssz)]).astype(np.int64)
            self.arena = HostArena(int(offs[-1]))
            for j, i in enumerate(self.streamed):
                view = self.arena.array[offs[j]:offs[j] + max(sizes[i], 16)]
                _fill_image(view, self.segs[i])
                self.host[i] = self.arena.tensor[offs[j]:offs[j] + max(sizes[i], 16)]
            cap = _up(max(max(sizes[i] for i in self.streamed), 16))
            self.slots = [torch.empty(cap, dtype=torch.uint8, device=self.dev) for _ in range(max(1, slots))]
            self.copy_stream = torch.cuda.Stream(self.dev)
            self._consumed = [None] * len(self.slots)
            self._pending: list = []      # (layer, slot, upload-done event), in upload order
            self._next_slot = 0

    # -- streamed pipeline ---------------------------------------------------------
    def _issue_upload(self, layer: int) -> None:
        slot = self._next_slot
        self._next_slot = (slot + 1) % len(self.slots)
        cs = self.copy_stream
        if self._consumed[slot] is not None:
            cs.wait_event(self._consumed[slot])
        src = self.host[layer]
        with torch.cuda.stream(cs):
            t0 = _mark(cs) if self.timeline is not None else None
            self.slots[slot][:src.numel()].copy_(src, non_blocking=True)
            if t0 is not None:
                self.timeline.append(("upload", layer, t0, _mark(cs)))
            ev = torch.cuda.Event()
            ev.record(cs)
        self.h2d_bytes += src.numel()
        self._pending.append((layer, slot, ev))

    def _take_image(self, i: int) -> tuple[torch.Tensor, int, object]:
        """(device image holding layer i, slot id or -1, event to wait on)."""
        if i in self.images:
            return self.images[i], -1, None
        if not self._pending or self._pending[0][0] != i:
            # out of step (first use, or a forward that stopped early): restart the ring at layer i
            self.copy_stream.synchronize()
            self._pending.clear()
            j0 = self._stream_pos[i]
            for j in range(min(len(self.slots), len(self.streamed))):
                self._issue_upload(self.streamed[(j0 + j) % len(self.streamed)])
        layer, slot, ev = self._pending.pop(0)
        return self.slots[slot], slot, ev

    def _release_image(self, slot: int, stream) -> None:
        if slot < 0:
            return
        done = torch.cuda.Event()
        done.record(stream)
        self._consumed[slot] = done
        last = self._pending[-1][0] if self._pending else self.streamed[-1]
        self._issue_upload(self.streamed[(self._stream_pos[last] + 1) % len(self.streamed)])

    # -- decode ----------------------------------------------------------------
    @staticmethod
    def _out_layout(segs: list[_Seg]) -> tuple[list[int], int]:
        offs, pos = [], 0
        for g in segs:
            offs.append(pos)
            pos += (g.ss.rows * g.ss.cols_decoded + 127) // 128 * 128
        return offs, pos

    @staticmethod
    def _desc(g: _Seg, base: torch.Tensor, e0: int, out: torch.Tensor):
        ds = _device.DeviceStream(packed=base[g.packed_off:g.packed_off + g.packed_cap], nbytes=g.packed_n,
                                  capacity=g.packed_cap, offset_base=0,
                                  offsets=base[g.offs_off:g.offs_off + 4 * max(g.n_chunks, 1)].view(torch.int32),
                                  chunk_nbytes=base[g.nbs_off:g.nbs_off + 4 * max(g.n_chunks, 1)].view(torch.int32),
                                  chunk_base=0)
        return _device.make_desc(ds, g.tables, g.ss.layer.encoded, e0, e0 + out.numel(), out, base[g.sm_off + e0:])

    def _layer_plan(self, i: int, slot: int, oset: int):
        """(descriptor array, name -> weight view) for decoding layer i from
        image `slot` (-1: its resident image) into output set `oset`."""
        key = (i, slot, oset)
        plan = self._desc_cache.get(key)
        if plan is None:
            segs = self.segs[i]
            base = self.images[i] if slot < 0 else self.slots[slot]
            buf = self._out_sets[oset]
            p = "model.layers.%d." % i
            d = (_lib.StreamDesc * max(1, len(segs)))()
            views = {}
            for j, (g, off) in enumerate(zip(segs, self._out_offs[i])):
                ss = g.ss
                o = buf[off:off + ss.rows * ss.cols_decoded]
                d[j] = self._desc(g, base, ss.elem_lo, o)
                views[g.key[len(p):]] = (o.view(ss.rows, ss.cols_decoded), ss)
            # q/k/v and gate/up decoded back to back: one projection each
            for joined, names in self.JOINS:
                parts = [views.get(n) for n in names]
                if all(v is not None and v[1].col_lo == 0 and v[1].cols == v[1].cols_decoded for v in parts):
                    t = self._adjacent([v[0] for v in parts])
                    if t is not None:
                        views[joined] = (t, None)
            plan = (d, views)
            self._desc_cache[key] = plan
        return plan

    def _decode_layer(self, i: int, stream, oset: int) -> dict:
        """Enqueues layer i's decode on `stream` into output set `oset`;
        returns name -> weight (views of the set)."""
        segs = self.segs[i]
        with torch.cuda.stream(stream):
            image, slot, ev = self._take_image(i)
            if ev is not None:
                stream.wait_event(ev)
            if self._set_free[oset] is not None and self.overlap:
                stream.wait_event(self._set_free[oset])
            descs, views = self._layer_plan(i, slot, oset)
            if segs:
                t0 = _mark(stream) if self.timeline is not None else None
                self.decoder.launch(descs, len(segs), max_ctas=self.decode_sms)
                if t0 is not None:
                    self.timeline.append(("decode", i, t0, _mark(stream)))
            self._release_image(slot, stream)
            W = {}
            for name, (o, ss) in views.items():
                W[name] = o if (ss is None or (ss.col_lo == 0 and ss.cols == ss.cols_decoded)) else \
                    o[:, ss.col_lo:ss.col_lo + ss.cols].contiguous()
        return W

    def begin_forward(self) -> None:
        if self.overlap:
            # the side stream starts from everything enqueued so far (and joins a graph capture)
            self._ahead.clear()
            self._set_free = [None] * len(self._out_sets)
            self._dec_stream.wait_stream(torch.cuda.current_stream(self.dev))

    def layer_weights(self, i: int) -> dict:
        compute = torch.cuda.current_stream(self.dev)
        if not self.overlap:
            W = self._decode_layer(i, compute, 0)
        else:
            ds = self._dec_stream
            # every op of layer i-1 is enqueued: its output set is free once they have run
            self._set_free[(i - 1) % 2] = self._event(compute)
            if i not in self._ahead:
                self._ahead[i] = (self._decode_layer(i, ds, i % 2), self._event(ds))
            W, ev = self._ahead.pop(i)
            compute.wait_event(ev)
            # the next layer decodes on the side stream while this one's projections run
            nxt = i + 1
            if nxt < self.n_layers:
                self._ahead[nxt] = (self._decode_layer(nxt, ds, nxt % 2), self._event(ds))
        p = "model.layers.%d." % i
        # norms, and projections the store kept raw (incompressible), are resident as-is
        for key in self.layer_keys[i]:
            if key[len(p):] not in W:
                W[key[len(p):]] = self.w[key]
        return W

    @staticmethod
    def _event(stream):
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev

    def head_logits(self, x: torch.Tensor) -> torch.Tensor:
        if self.head is None:
            return super().head_logits(x)
        g, image = self.head
        ss = g.ss
        rows, cols = ss.rows, ss.cols
        out = torch.empty(x.shape[0], rows, dtype=x.dtype, device=self.dev)
        blk = self.head_block_rows
        for r0 in range(0, rows, blk):
            r1 = min(rows, r0 + blk)
            key = ("head", r0)
            plan = self._desc_cache.get(key)
            if plan is None:
                w = self._head_buf[:(r1 - r0) * ss.cols_decoded]
                d = (_lib.StreamDesc * 1)()
                d[0] = self._desc(g, image, ss.elem_lo + r0 * ss.cols_decoded, w)
                plan = (d, w.view(r1 - r0, ss.cols_decoded)[:, ss.col_lo:ss.col_lo + cols])
                self._desc_cache[key] = plan
            d, wv = plan
            self.decoder.launch(d, 1)
            out[:, r0:r1] = self._proj(x, wv)
        return out

    def decode_bytes_per_forward(self) -> int:
        """Algorithmic bytes one forward's decodes move on this rank:
        sign/mantissa + packed stream + 4-byte chunk offsets + the 32 KiB
        first-level table per tensor, plus 2 bytes per BF16 written."""
        total = 0
        segs = [g for layer in self.segs for g in layer] + ([self.head[0]] if self.head is not None else [])
        for g in segs:
            n = g.ss.rows * g.ss.cols_decoded
            total += n + g.packed_n + 4 * g.n_chunks + 32768 + 2 * n
        return total

    def weights_per_forward(self) -> int:
        """Weights one forward's projections read on this rank (decoded
        elements of every layer shard and of the head shard)."""
        segs = [g for layer in self.segs for g in layer] + ([self.head[0]] if self.head is not None else [])
        return sum(g.ss.rows * g.ss.cols_decoded for g in segs)

    def h2d_bytes_per_forward(self) -> int:
        return sum(int(h.numel()) for h in self.host.values())

    def close(self) -> None:
        super().close()
        if self.streamed:
            self.copy_stream.synchronize()
            torch.cuda.synchronize(self.dev)
            self.slots = []
            self.host = {}
            self.arena.close()
            self.streamed = []


class HostRows:
    """Embedding rows gathered on the host from a page-locked table and
    uploaded per call (the row-gather embedding; the table never occupies
    device memory)."""

    def __init__(self, table: torch.Tensor, device):
        self.table = table.pin_memory() if torch.cuda.is_available() else table
        self.device = device

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        rows = self.table.index_select(0, ids.to("cpu"))
        return rows.to(self.device, non_blocking=False)


def load_tp_decoder(store_dir, hf_cfg, world: int = 1, rank: int = 0, group=None, device="cuda",
                    resident: str = "decoded", **kw) -> TPDecoder:
    """Builds rank `rank`'s decoder from a compressed store. Projection
    shards are cut from the chunk streams on the host and then
      resident="decoded":    decoded once into BF16 shards in HBM;
      resident="compressed": kept compressed in HBM, decoded per forward;
      resident="streamed":   kept compressed in page-locked host memory and
                             copied to the device one layer at a time.
    Norms are replicated; the head is split by vocabulary (kept compressed
    unless decoded); an untied row-gather embedding stays in host memory
    when streamed. collective="oneshot" (default) sums the row-parallel
    projections with the one-shot NVLink all-reduce on GPU ranks (NCCL
    otherwise, and for sums above its buffer); "nccl" keeps NCCL. Extra
    keywords go to CompressedTPDecoder."""
    from .compressed_store import decompress_layer_gpu
    if resident not in ("decoded", "compressed", "streamed"):
        raise ValueError("resident must be 'decoded', 'compressed' or 'streamed'")
    collective = kw.pop("collective", "oneshot")
    if collective not in ("oneshot", "nccl"):
        raise ValueError("collective must be 'oneshot' or 'nccl'")
    store = pathlib.Path(store_dir)
    manifest = json.loads((store / "manifest.json").read_text())
    dev = _device.cuda_device(device)
    weights: dict = {}
    streams: dict = {}
    keep_compressed = resident in ("compressed", "streamed")
    with BinaryWeightReader(store / "weights.bin") as reader:
        for key, meta in manifest["tensors"].items():
            blobs = {n: reader.read(ref) for n, ref in meta["blobs"].items()}
            if meta.get("row_gather"):
                # untied embedding stored raw: replicated rows
                from .streaming_engine import _raw_tensor
                table = _raw_tensor(meta, blobs["raw"]).reshape(meta["shape"])
                weights[key] = HostRows(table, dev) if resident == "streamed" else table.to(dev)
                continue
            if not meta["compressed"]:
                # stored raw (incompressible): shard by slicing
                from .streaming_engine import _raw_tensor
                t = _raw_tensor(meta, blobs["raw"]).reshape(meta["shape"])
                kind = shard_kind(key)
                if kind == "col":
                    r0, r1 = _split(t.shape[0], world, rank)
                    t = t[r0:r1]
                elif kind == "row":
                    c0, c1 = _split(t.shape[1], world, rank)
                    t = t[:, c0:c1]
                weights[key] = t.contiguous().to(dev)
                continue
            from .streaming_engine import _encoded_from_arrays
            layer = _encoded_from_arrays(meta, blobs)
            kind = shard_kind(key)
            if kind == "rep":
                weights[key] = decompress_layer_gpu(layer, device=dev)
                continue
            ss = shard_stream(layer, kind, world, rank)
            if keep_compressed and (key.startswith("model.layers.") or key == "lm_head.weight"):
                streams[key] = ss
                weights[key] = None
                continue
            weights[key] = ss.finish(decompress_layer_gpu(ss.layer, device=dev))
    if "lm_head.weight" not in weights and not getattr(hf_cfg, "tie_word_embeddings", False):
        raise RuntimeError("store has no lm_head.weight and the model is not tied")
    if keep_compressed:
        dec = CompressedTPDecoder(hf_cfg, weights, streams, world, rank, group, dev,
                                  mode="streamed" if resident == "streamed" else "compressed", **kw)
    else:
        dec = TPDecoder(hf_cfg, weights, world, rank, group, dev, fused=kw.get("fused", True))
    if collective == "oneshot":
        dec.use_oneshot_allreduce()
    return dec
