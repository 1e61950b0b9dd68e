"""Tensor-parallel HiF4 W4A4 prefill over NCCL: the multi-GPU form of the two hot paths.

Megatron-style sharding, one process per GPU (``torch.distributed``, backend ``nccl``):

* column-parallel projections (Qwen3 q/k/v and gate/up; Wan q/k/v and ffn.0) keep a
  contiguous slice of output rows. Their input is replicated, so K1 quantizes the whole
  input with its full HiSQ rotation -- bit-identical to the single-GPU module -- and the
  GEMM runs on the local rows. Projections that read the same normalized input share
  one rotation and one K1 launch (the reference's ``hisq_rotation_source`` sharing
  ``"norm"``, ``hisq_rotation.py:204-212``) and one GEMM over their concatenated rows.
* row-parallel projections (o_proj, down_proj; Wan o and ffn.2) keep the input columns
  of their shard and end in one NCCL all-reduce (sum, bf16) of the partial outputs. The
  rotation of a row-parallel input must stay inside the shard: it uses the reference's
  ``"signs"`` construction (``restrict_hisq_rotation``, ``hisq_rotation.py:156-167``:
  sign flips, no permutation) with 64-channel Hadamard blocks, so HiF4 groups and
  rotation blocks never straddle a shard at 1/2/4/8 GPUs.

Only the GEMM accumulation order depends on the number of ranks (partial sums meet in
the all-reduce); every quantized activation and weight code is the same at any TP size.

With more than one rank the models run sequence-parallel by default (``SeqLayout``): the
residual stream between projections is sharded by rows, so the norms and the readers'
quantization run on 1/N of the rows instead of on every rank in full; the column-parallel
inputs are all-gathered as packed HiF4 codes (0.5625 bytes per value instead of bf16's
2) and the row-parallel outputs are reduce-scattered instead of all-reduced, one chunk of
rows at a time (``sp_chunks``; one by default: the persistent GEMMs and the attention
hold every SM, so a collective cannot run beside them and more chunks only add calls).
Per row the arithmetic is the all-reduce path's; at two ranks the outputs are the same
bits.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch
from torch import nn

from . import ops
from .hisq_rotation import derive_hisq_rotation, hisq_rotation_source, restrict_hisq_rotation

HIF4_GROUP = 64


@dataclass
class TPGroup:
    """This rank's place in the tensor-parallel group (``world == 1``: no collective)."""

    rank: int = 0
    world: int = 1
    group: object | None = None
    # when a list: every collective appends (start event, end event, bytes, kind), recorded
    # on the stream it runs on -- the measurement of the collectives' share of a step
    timer: list | None = None
    # SMs the persistent GEMMs leave free during a sequence-parallel forward, for the NCCL
    # kernels of the chunked collectives that run beside them (0: GEMMs on every SM)
    gemm_sm_reserve: int = 0

    def gemm_sms(self, device: torch.device):
        """Context: the GEMMs inside run on all but ``gemm_sm_reserve`` SMs."""
        import contextlib

        if self.gemm_sm_reserve <= 0:
            return contextlib.nullcontext()

        @contextlib.contextmanager
        def ctx():
            total = torch.cuda.get_device_properties(device).multi_processor_count
            ops.set_gemm_sm_target(max(2, total - self.gemm_sm_reserve))
            try:
                yield
            finally:
                ops.set_gemm_sm_target(0)

        return ctx()

    def shard(self, n: int, unit: int) -> tuple[int, int]:
        """(start, size) of this rank's even share of ``n`` items in whole ``unit``s."""
        if n % (self.world * unit):
            raise ValueError(f"{n} does not split into {self.world} shards of whole {unit}-blocks")
        size = n // self.world
        return self.rank * size, size

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist

            self._timed(lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group),
                        t.numel() * t.element_size(), "all_reduce")
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """``[world, *t.shape]``: every rank's ``t`` in rank order."""
        if self.world == 1:
            return t.unsqueeze(0)
        out = torch.empty((self.world, *t.shape), dtype=t.dtype, device=t.device)
        self.all_gather_into(out.view(-1, *t.shape[1:]) if t.dim() else out, t)
        return out

    def _timed(self, call, nbytes: int, kind: str) -> None:
        if self.timer is None or not torch.cuda.is_available():
            call()
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        self.timer.append((e0, e1, nbytes, kind))

    def all_gather_into(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """``out [world * n, ...]`` <- every rank's ``t [n, ...]`` in rank order (NCCL
        all-gather; ``out`` must be contiguous)."""
        if self.world == 1:
            out.copy_(t)
            return out
        import torch.distributed as dist

        t = t.contiguous()
        self._timed(lambda: dist.all_gather_into_tensor(out, t, group=self.group), out.numel() * out.element_size(),
                    "all_gather")
        return out

    def reduce_scatter(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """``out [n, ...]`` <- rows ``rank * n .. rank * n + n - 1`` of the sum over ranks of
        ``t [world * n, ...]`` (NCCL reduce-scatter, sum)."""
        if self.world == 1:
            out.copy_(t)
            return out
        import torch.distributed as dist

        t = t.contiguous()
        self._timed(lambda: dist.reduce_scatter_tensor(out, t, op=dist.ReduceOp.SUM, group=self.group),
                    t.numel() * t.element_size(), "reduce_scatter")
        return out

    def comm_stream(self, device: torch.device) -> torch.cuda.Stream:
        """The side stream the chunked collectives run on (one per rank and device)."""
        key = ("stream", device.index)
        cache = self.__dict__.setdefault("_streams", {})
        if key not in cache:
            cache[key] = torch.cuda.Stream(device=device)
        return cache[key]


@dataclass(frozen=True)
class SeqLayout:
    """Sequence-parallel row layout of a ``[rows, hidden]`` activation: the rows are cut
    into ``chunks`` equal chunks and every chunk into ``world`` equal pieces; rank ``r``
    holds piece ``r`` of every chunk, in chunk order (its shard, ``[chunks * piece,
    hidden]``). A reduce-scatter of chunk ``c`` of a row-parallel output lands in piece
    ``c`` of each rank's shard, and an all-gather of piece ``c`` rebuilds chunk ``c`` in
    row order, so the collectives of one chunk can overlap the GEMM of the next."""

    rows: int
    world: int
    rank: int
    chunks: int

    @property
    def chunk_rows(self) -> int:
        return self.rows // self.chunks

    @property
    def piece(self) -> int:
        return self.rows // (self.chunks * self.world)

    @property
    def shard_rows(self) -> int:
        return self.chunks * self.piece

    def chunk(self, c: int) -> slice:
        return slice(c * self.chunk_rows, (c + 1) * self.chunk_rows)

    def piece_of_shard(self, c: int) -> slice:
        return slice(c * self.piece, (c + 1) * self.piece)

    def owned(self, device: torch.device | str = "cpu") -> torch.Tensor:
        """Row indices of this rank's shard, in shard order."""
        base = torch.arange(self.chunks, device=device) * self.chunk_rows + self.rank * self.piece
        return (base[:, None] + torch.arange(self.piece, device=device)[None, :]).reshape(-1)

    def locate(self, row: int) -> tuple[int, int]:
        """(rank, index in that rank's shard) of ``row``."""
        c, within = divmod(row, self.chunk_rows)
        r, i = divmod(within, self.piece)
        return r, c * self.piece + i


def seq_layout(rows: int, tp: TPGroup, max_chunks: int = 4) -> SeqLayout | None:
    """The layout with the most chunks (at most ``max_chunks``) that splits ``rows`` evenly,
    or None when ``rows`` does not divide by the TP size (the replicated path then runs)."""
    for chunks in range(max_chunks, 0, -1):
        if rows % (chunks * tp.world) == 0:
            return SeqLayout(rows, tp.world, tp.rank, chunks)
    return None


def sp_gather_rows(tp: TPGroup, lay: SeqLayout, shard: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather of a sequence-parallel shard back to ``[rows, ...]`` in row order, one
    collective per chunk."""
    if out is None:
        out = torch.empty((lay.rows, *shard.shape[1:]), dtype=shard.dtype, device=shard.device)
    for c in range(lay.chunks):
        tp.all_gather_into(out[lay.chunk(c)], shard[lay.piece_of_shard(c)])
    return out


def sp_reduce_scatter_rows(tp: TPGroup, lay: SeqLayout, full: torch.Tensor,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Reduce-scatter of a row-parallel ``[rows, ...]`` partial into this rank's shard,
    one collective per chunk."""
    if out is None:
        out = torch.empty((lay.shard_rows, *full.shape[1:]), dtype=full.dtype, device=full.device)
    for c in range(lay.chunks):
        tp.reduce_scatter(out[lay.piece_of_shard(c)], full[lay.chunk(c)])
    return out


def _seed(*parts: object) -> int:
    """Deterministic 63-bit seed of a weight's name (identical on every rank and TP size)."""
    return int.from_bytes(hashlib.sha256("::".join(map(str, parts)).encode()).digest()[:8], "little") >> 1


def random_weight(shape: tuple[int, int], seed: int, device: torch.device, std: float = 0.02) -> torch.Tensor:
    """``N(0, std)`` weight drawn in full on ``device`` (every rank draws the same matrix)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device) * std).to(torch.bfloat16)


@dataclass
class Rotation:
    """Input rotation of a projection as K1 takes it (``signs`` None: no rotation)."""

    signs: torch.Tensor | None = None
    permutation: torch.Tensor | None = None
    block: int = 0

    def to(self, device: torch.device) -> "Rotation":
        return Rotation(None if self.signs is None else self.signs.to(device),
                        None if self.permutation is None else self.permutation.to(device), self.block)


def column_rotation(name: str, k: int, *, seed: int, block: int, sharing: str = "norm") -> Rotation:
    """Full HiSQ rotation of a column-parallel projection's (replicated) input."""
    source, source_seed = hisq_rotation_source(name, sharing, seed=seed, global_seed=seed)
    rot = derive_hisq_rotation(source, k, seed=source_seed, block_size=block)
    return Rotation(rot.signs, rot.permutation, block)


def row_rotation(name: str, k: int, tp: TPGroup, *, seed: int, block: int = HIF4_GROUP) -> Rotation:
    """Shard-local ``"signs"`` rotation of a row-parallel projection's input slice."""
    rot = restrict_hisq_rotation(derive_hisq_rotation(name, k, seed=seed, block_size=block), "signs")
    start, size = tp.shard(k, block)
    return Rotation(rot.signs[start:start + size].clone(), None, block)


class TPHiF4Linear(nn.Module):
    """One rank's shard of a HiF4 W4A4 projection (or a plain bf16 one).

    ``weight`` is the local ``[n_local, k_local]`` bf16 slice; when ``quantize`` is set it
    is RTN-quantized to the HiF4 grid here (groups of 64 along k stay whole in a slice)
    and the input goes through K1 with ``rotation``. ``reduce`` makes it row-parallel.
    """

    def __init__(self, weight: torch.Tensor, *, rotation: Rotation | None, quantize: bool, levels: str = "123",
                 bias: torch.Tensor | None = None, reduce: TPGroup | None = None) -> None:
        super().__init__()
        if quantize:
            weight = ops.hif4_quantize(weight.to(torch.bfloat16), levels=levels)[0]
        self.register_buffer("weight", weight.to(torch.bfloat16).contiguous())
        self.register_buffer("bias", None if bias is None else bias.to(torch.bfloat16).contiguous())
        self.rotation = (rotation or Rotation()).to(weight.device)
        self.quantize = quantize
        self.levels = levels
        self.reduce = reduce

    def quantize_input(self, x: torch.Tensor) -> torch.Tensor:
        if not self.quantize:
            return x
        r = self.rotation
        return ops.hif4_quantize(x, levels=self.levels, signs=r.signs, permutation=r.permutation,
                                 rot_block=r.block if r.signs is not None else None)[0]

    # row chunks of a row-parallel GEMM whose all-reduce overlaps the next chunk's GEMM
    overlap_chunks = 4
    overlap_min_rows = 4096

    def activate_and_quantize(self, x: torch.Tensor, act: str) -> torch.Tensor:
        """The input ``act(x)`` ("swiglu" on gate|up, or "gelu_tanh") quantized: in one pass
        (``ops.hif4_quantize_act``) for a quantized projection with a signs-only rotation,
        else the activation kernel then :meth:`quantize_input` -- the same values."""
        r = self.rotation
        if self.quantize and r.signs is not None and r.permutation is None and 8 <= r.block <= 256:
            return ops.hif4_quantize_act(x, act, levels=self.levels, signs=r.signs, rot_block=r.block)[0]
        return self.quantize_input(ops.silu_mul(x) if act == "swiglu" else ops.gelu_tanh(x))

    def norm_and_quantize(self, x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
        """The input ``rms_norm(x, weight, eps)`` (``weight=None``: ``layer_norm(x, eps)``)
        quantized: in one pass (``ops.hif4_quantize_rms_norm``: the norm inside K1, nothing
        written between) for a quantized projection with a rotation K1 v4 takes, else the
        norm kernel then :meth:`quantize_input` -- the same values."""
        r = self.rotation
        if self.quantize and r.signs is not None and ops.rms_norm_quantize_supported(x.shape[-1], r.block):
            return ops.hif4_quantize_rms_norm(x, weight, eps, levels=self.levels, signs=r.signs,
                                              permutation=r.permutation, rot_block=r.block)[0]
        h = ops.layer_norm(x, eps) if weight is None else ops.rms_norm(x, weight, eps)
        return self.quantize_input(h)

    def forward(self, x: torch.Tensor, *, quantized: bool = False, residual: torch.Tensor | None = None,
                act: str | None = None, norm: tuple[torch.Tensor, float] | None = None) -> torch.Tensor:
        """``residual + linear(act(x))``: ``act`` ("swiglu" / "gelu_tanh") is applied to the
        input first, fused into its quantization where possible; ``norm = (weight, eps)``
        applies the RMSNorm to the input first, likewise fused; with ``residual`` on one
        rank the add is in the GEMM epilogue (the same bits as the separate bf16 add),
        row-parallel ranks add after the all-reduce."""
        if norm is not None:
            xq = self.norm_and_quantize(x, *norm)
        elif act is not None:
            xq = self.activate_and_quantize(x, act)
        else:
            xq = x if quantized else self.quantize_input(x)
        tp = self.reduce
        if tp is None or tp.world == 1:
            return ops.gemm_bf16(xq, self.weight, self.bias, residual=residual)
        y = self._row_parallel(xq)
        return y if residual is None else residual + y

    # ------------------------------------------------ sequence-parallel forms
    def sp_column(self, x_shard: torch.Tensor, lay: SeqLayout, tp: TPGroup,
                  norm: tuple[torch.Tensor | None, float] | None = None) -> torch.Tensor:
        """Column-parallel projection of a sequence-parallel input: ``x_shard`` holds this
        rank's rows (``lay``); the norm (``norm = (weight, eps)``, ``weight=None``: the
        affine-free LayerNorm) and the input quantization run on the shard only, the
        quantized rows are all-gathered -- as packed HiF4 codes and meta words (0.5625
        bytes per value) when the norm is fused into K1 -- expanded back to the bf16
        operand (the same values K1 would have written) and multiplied, chunk by chunk, so
        chunk ``c + 1`` moves over NVLink while chunk ``c`` is expanded and multiplied.
        Returns the ``[rows, n_local]`` output."""
        dev = x_shard.device
        k = x_shard.shape[1]
        r = self.rotation
        packed = (self.quantize and norm is not None and r.signs is not None
                  and ops.rms_norm_quantize_supported(k, r.block))
        if packed:
            codes = torch.empty((x_shard.shape[0], k // 2), dtype=torch.uint8, device=dev)
            _, meta = ops.hif4_quantize_rms_norm(x_shard, norm[0], norm[1], levels=self.levels, signs=r.signs,
                                                 permutation=r.permutation, rot_block=r.block, want_meta=True,
                                                 want_qdq=False, codes_out=codes)
            shards = [codes, meta]
        elif norm is not None:
            h = ops.layer_norm(x_shard, norm[1]) if norm[0] is None else ops.rms_norm(x_shard, norm[0], norm[1])
            shards = [self.quantize_input(h)]
        else:
            shards = [self.quantize_input(x_shard)]
        fulls = [torch.empty((lay.rows, *t.shape[1:]), dtype=t.dtype, device=dev) for t in shards]
        y = torch.empty((lay.rows, self.weight.shape[0]), dtype=torch.bfloat16, device=dev)
        compute = torch.cuda.current_stream(dev)
        comm = tp.comm_stream(dev)
        comm.wait_stream(compute)  # the shard's quantized rows are written
        for t in shards + fulls:
            t.record_stream(comm)

        def consume(c: int) -> None:
            ev = torch.cuda.Event()
            ev.record(comm)
            compute.wait_event(ev)
            rows = lay.chunk(c)
            if packed:
                a = torch.empty((lay.chunk_rows, k), dtype=torch.bfloat16, device=dev)
                ops.hif4_dequantize(fulls[0][rows], fulls[1][rows], k, out=a)
            else:
                a = fulls[0][rows]
            ops.gemm_bf16(a, self.weight, self.bias, out=y[rows])

        for c in range(lay.chunks):
            with torch.cuda.stream(comm):
                for src, dst in zip(shards, fulls):
                    tp.all_gather_into(dst[lay.chunk(c)], src[lay.piece_of_shard(c)])
            consume(c)
        return y

    def sp_row(self, xq: torch.Tensor, residual: torch.Tensor, lay: SeqLayout, tp: TPGroup) -> torch.Tensor:
        """Row-parallel projection into a sequence-parallel residual stream: the GEMM of
        the quantized input ``xq [rows, k_local]`` chunk by chunk, each chunk's partial
        output reduce-scattered (NCCL, sum in bf16) while the next chunk multiplies, and
        added to this rank's residual rows. Returns the new ``[shard_rows, hidden]``
        residual (the same sums and bf16 adds as the all-reduce path's rows)."""
        dev = xq.device
        n = self.weight.shape[0]
        out = torch.empty_like(residual)
        compute = torch.cuda.current_stream(dev)
        comm = tp.comm_stream(dev)
        residual.record_stream(comm)
        out.record_stream(comm)
        for c in range(lay.chunks):
            part = torch.empty((lay.chunk_rows, n), dtype=torch.bfloat16, device=dev)
            ops.gemm_bf16(xq[lay.chunk(c)], self.weight, self.bias, out=part)
            comm.wait_stream(compute)
            part.record_stream(comm)
            with torch.cuda.stream(comm):
                red = torch.empty((lay.piece, n), dtype=torch.bfloat16, device=dev)
                tp.reduce_scatter(red, part)
                p = lay.piece_of_shard(c)
                torch.add(residual[p], red, out=out[p])
        compute.wait_stream(comm)
        return out

    def _row_parallel(self, xq: torch.Tensor) -> torch.Tensor:
        tp = self.reduce
        rows = xq.shape[0]
        if rows < self.overlap_min_rows:
            return tp.all_reduce_(ops.gemm_bf16(xq, self.weight, self.bias))
        # chunk i's all-reduce (side stream, NCCL over NVLink) runs while chunk i + 1's GEMM
        # computes; the sums are those of one all-reduce of the whole output
        y = torch.empty((rows, self.weight.shape[0]), dtype=torch.bfloat16, device=xq.device)
        compute = torch.cuda.current_stream(xq.device)
        comm = tp.comm_stream(xq.device)
        step = -(-rows // self.overlap_chunks)
        step = (step + 127) // 128 * 128
        for r0 in range(0, rows, step):
            part = y[r0:r0 + step]
            ops.gemm_bf16(xq[r0:r0 + step], self.weight, self.bias, out=part)
            comm.wait_stream(compute)
            with torch.cuda.stream(comm):
                tp.all_reduce_(part)
                part.record_stream(comm)
        compute.wait_stream(comm)
        return y


# ---------------------------------------------------------------- elementwise glue (torch)
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``Qwen3RMSNorm``: fp32 mean of squares, rsqrt, cast back, times the weight."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype)


def rope_tables(seq: int, dim: int, theta: float, device: torch.device, dtype=torch.bfloat16):
    """cos/sin ``[seq, dim]`` of HF's default rotary embedding (``rotate_half`` layout)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    freqs = torch.outer(torch.arange(seq, device=device, dtype=torch.float32), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x [B, S, H, D]``: ``x * cos + rotate_half(x) * sin`` (HF ``apply_rotary_pos_emb``)."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[None, :, None, :] + rot * sin[None, :, None, :]


# ---------------------------------------------------------------- Qwen3 tensor-parallel prefill
@dataclass
class Qwen3TPConfig:
    """Qwen3-32B shapes; smaller values for tests."""

    hidden: int = 5120
    layers: int = 64
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 25600
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    bf16_layers: tuple[int, ...] = (39, 40, 42, 45, 46)
    levels: str = "123"
    hisq_seed: int = 17
    column_block: int = 1024
    seed: int = 0

    def flops(self, batch: int, seq: int) -> dict[str, float]:
        """Algorithmic FLOPs of one prefill (last-token logits only)."""
        t = batch * seq
        per_layer = self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim \
            + self.heads * self.head_dim * self.hidden + 3 * self.hidden * self.ffn
        linear = 2.0 * t * per_layer * self.layers
        attention = 4.0 * self.head_dim * self.heads * batch * seq * (seq + 1) / 2.0 * self.layers
        lm_head = 2.0 * batch * self.hidden * self.vocab
        return {"linear": linear, "attention": attention, "lm_head": lm_head,
                "total": linear + attention + lm_head}


def qwen3_shard_slices(cfg: Qwen3TPConfig, tp: TPGroup) -> dict[str, slice]:
    """This rank's rows of q / k,v (column-parallel), input columns of o_proj and the FFN
    channels (gate/up rows, down_proj columns) -- head-aligned and 64-aligned."""
    if cfg.heads % tp.world or cfg.kv_heads % tp.world:
        raise ValueError("heads and kv_heads must divide by the TP size")
    d = cfg.head_dim
    hq, hkv = cfg.heads // tp.world, cfg.kv_heads // tp.world
    f0, fl = tp.shard(cfg.ffn, HIF4_GROUP)
    q = slice(tp.rank * hq * d, (tp.rank + 1) * hq * d)
    return {"q_rows": q, "kv_rows": slice(tp.rank * hkv * d, (tp.rank + 1) * hkv * d), "o_cols": q,
            "ffn": slice(f0, f0 + fl)}


@dataclass
class _Qwen3Layer:
    qkv: TPHiF4Linear
    o: TPHiF4Linear
    gate_up: TPHiF4Linear
    down: TPHiF4Linear
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    heads: int
    kv_heads: int
    ffn: int


class Qwen3TPPrefill(nn.Module):
    """One rank of a Qwen3 prefill forward with HiF4 W4A4 projections and HiF4 QK/PV
    attention (``qwen3._attention_forward``, ``qwen3.py:56-172``, with the decoder layer
    of HF ``Qwen3DecoderLayer``), random-initialized ``N(0, 0.02)`` weights, RTN HiF4.

    Attention per rank: ``heads / world`` query heads and ``kv_heads / world`` KV heads,
    the post-RoPE Hadamard over head_dim with HiF4 Q/K/V (K4) and the HiF4 attention
    kernel (K5, causal, P-Reordering). Layers in ``bf16_layers`` keep bf16 projections.
    The logits are those of the last position of every sequence. ``trace``, when set,
    is called as ``trace(stage, layer, tensor)`` at every stage boundary (tests compare
    each stage with the oracle on that stage's own input: 4-bit quantization is
    discontinuous, so differences between two implementations are only comparable one
    stage at a time).
    """

    def __init__(self, cfg: Qwen3TPConfig, tp: TPGroup, device: torch.device) -> None:
        super().__init__()
        self.cfg, self.tp, self.device = cfg, tp, device
        self.trace = None
        # the residual adds in the o_proj / down_proj GEMM epilogues (off while a trace hook
        # needs the projections' own outputs)
        self.fuse_residual = True
        # with more than one rank: the residual stream sharded by rows, reduce-scatter and
        # all-gather of packed codes instead of all-reduces (off while a trace hook is set),
        # in up to sp_chunks row chunks (one: the fewest collectives, fastest measured at TP 8)
        self.sequence_parallel = True
        self.sp_chunks = 1
        d = cfg.head_dim
        sl = qwen3_shard_slices(cfg, tp)
        hq, hkv = cfg.heads // tp.world, cfg.kv_heads // tp.world
        q_rows, kv_rows, o_cols, ffn = sl["q_rows"], sl["kv_rows"], sl["o_cols"], sl["ffn"]
        fl = ffn.stop - ffn.start
        self.embed = random_weight((cfg.vocab, cfg.hidden), _seed(cfg.seed, "embed"), device)
        self.lm_head = random_weight((cfg.vocab, cfg.hidden), _seed(cfg.seed, "lm_head"), device)
        self.final_norm = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device)
        self.layers: list[_Qwen3Layer] = []
        for i in range(cfg.layers):
            quant = i not in cfg.bf16_layers
            name = f"model.layers.{i}"

            def w(proj: str, n: int, k: int) -> torch.Tensor:
                return random_weight((n, k), _seed(cfg.seed, name, proj), device)

            wq = w("self_attn.q_proj", cfg.heads * d, cfg.hidden)[q_rows]
            wk = w("self_attn.k_proj", cfg.kv_heads * d, cfg.hidden)[kv_rows]
            wv = w("self_attn.v_proj", cfg.kv_heads * d, cfg.hidden)[kv_rows]
            wo = w("self_attn.o_proj", cfg.hidden, cfg.heads * d)[:, o_cols]
            wg = w("mlp.gate_proj", cfg.ffn, cfg.hidden)[ffn]
            wu = w("mlp.up_proj", cfg.ffn, cfg.hidden)[ffn]
            wd = w("mlp.down_proj", cfg.hidden, cfg.ffn)[:, ffn]
            rot = dict(seed=cfg.hisq_seed, block=cfg.column_block)
            layer = _Qwen3Layer(
                qkv=TPHiF4Linear(torch.cat([wq, wk, wv]), quantize=quant, levels=cfg.levels,
                                 rotation=column_rotation(f"{name}.self_attn.q_proj", cfg.hidden, **rot)),
                o=TPHiF4Linear(wo, quantize=quant, levels=cfg.levels, reduce=tp,
                               rotation=row_rotation(f"{name}.self_attn.o_proj", cfg.heads * d, tp,
                                                     seed=cfg.hisq_seed)),
                gate_up=TPHiF4Linear(torch.cat([wg, wu]), quantize=quant, levels=cfg.levels,
                                     rotation=column_rotation(f"{name}.mlp.gate_proj", cfg.hidden, **rot)),
                down=TPHiF4Linear(wd, quantize=quant, levels=cfg.levels, reduce=tp,
                                  rotation=row_rotation(f"{name}.mlp.down_proj", cfg.ffn, tp, seed=cfg.hisq_seed)),
                input_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device),
                post_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device),
                q_norm=torch.ones(d, dtype=torch.bfloat16, device=device),
                k_norm=torch.ones(d, dtype=torch.bfloat16, device=device),
                heads=hq, kv_heads=hkv, ffn=fl,
            )
            self.layers.append(layer)

    def _t(self, stage: str, index: int, t: torch.Tensor) -> torch.Tensor:
        if self.trace is not None:
            self.trace(stage, index, t)
        return t

    def _attention(self, layer: _Qwen3Layer, h: torch.Tensor, batch: int, seq: int, cos, sin,
                   index: int = 0, residual: torch.Tensor | None = None,
                   norm: tuple[torch.Tensor, float] | None = None) -> torch.Tensor:
        """``h`` is the normalized input, or with ``norm`` the raw one (the norm is then
        fused into the qkv input quantization)."""
        if norm is None:
            qkv = self._t("qkv", index, layer.qkv(self._t("input_norm", index, h)))  # [T, (hq + 2 hkv) d]
        else:
            qkv = self._t("qkv", index, layer.qkv(h, norm=norm))
        out = self._attend(layer, qkv, batch, seq, cos, sin, index)
        return self._t("o", index, layer.o(out, residual=residual))

    def _attend(self, layer: _Qwen3Layer, qkv: torch.Tensor, batch: int, seq: int, cos, sin,
                index: int = 0) -> torch.Tensor:
        """The attention of the rank's heads from the qkv projection's output ``[T, (hq + 2
        hkv) d]``; returns ``[T, hq d]`` (the o_proj input)."""
        cfg, d = self.cfg, self.cfg.head_dim
        nq, nk = layer.heads * d, layer.kv_heads * d
        # q_norm/k_norm, RoPE, Hadamard and HiF4 in one K4 pass per operand
        q = qkv[:, :nq].view(batch, seq, layer.heads, d).transpose(1, 2)
        k = qkv[:, nq:nq + nk].view(batch, seq, layer.kv_heads, d).transpose(1, 2)
        v = qkv[:, nq + nk:].view(batch, seq, layer.kv_heads, d).transpose(1, 2)
        qd = self._t("qd", index, ops.qk_norm_rope_prep(q, norm_weight=layer.q_norm, eps=cfg.eps, cos=cos, sin=sin,
                                                        levels=cfg.levels))
        kd = self._t("kd", index, ops.qk_norm_rope_prep(k, norm_weight=layer.k_norm, eps=cfg.eps, cos=cos, sin=sin,
                                                        levels=cfg.levels))
        vd = self._t("vd", index, ops.qk_prep(v, levels=cfg.levels, rotate=False)[0])
        out = ops.hif4_attention(qd, kd, vd, scale=d ** -0.5, causal=True, p_levels=cfg.levels,
                                 quantized_normalizer=True)  # [B, S, hq, d]
        return self._t("attention", index, out).view(batch * seq, nq)

    def seq_layout(self, batch: int, seq: int) -> SeqLayout | None:
        """The sequence-parallel layout the forward uses (None: the replicated path)."""
        if not self.sequence_parallel or self.tp.world == 1 or self.trace is not None:
            return None
        return seq_layout(batch * seq, self.tp, self.sp_chunks)

    def _forward_sp(self, input_ids: torch.Tensor, lay: SeqLayout) -> torch.Tensor:
        """Sequence-parallel forward: the residual stream is sharded by rows (``lay``), the
        norms and the column-parallel inputs' quantization run on the shard and the packed
        codes are all-gathered (:meth:`TPHiF4Linear.sp_column`); the row-parallel outputs
        are reduce-scattered into the shard (:meth:`TPHiF4Linear.sp_row`). The same
        per-row arithmetic as the all-reduce path: at two ranks the logits are the same
        bits."""
        with self.tp.gemm_sms(self.device):
            return self._forward_sp_layers(input_ids, lay)

    def _forward_sp_layers(self, input_ids: torch.Tensor, lay: SeqLayout) -> torch.Tensor:
        cfg, tp = self.cfg, self.tp
        batch, seq = input_ids.shape
        cos, sin = rope_tables(seq, cfg.head_dim, cfg.rope_theta, self.device)
        x = torch.nn.functional.embedding(input_ids.reshape(-1)[lay.owned(self.device)], self.embed)
        for layer in self.layers:
            qkv = layer.qkv.sp_column(x, lay, tp, norm=(layer.input_norm, cfg.eps))
            att = self._attend(layer, qkv, batch, seq, cos, sin)
            x = layer.o.sp_row(layer.o.quantize_input(att), x, lay, tp)
            gu = layer.gate_up.sp_column(x, lay, tp, norm=(layer.post_norm, cfg.eps))
            x = layer.down.sp_row(layer.down.activate_and_quantize(gu, "swiglu"), x, lay, tp)
        # the last position of each sequence, from the rank that holds it (the others add zeros)
        last = torch.zeros((batch, cfg.hidden), dtype=torch.bfloat16, device=self.device)
        for b in range(batch):
            owner, i = lay.locate(b * seq + seq - 1)
            if owner == tp.rank:
                last[b] = x[i]
        tp.all_reduce_(last)
        return torch.nn.functional.linear(rms_norm(last, self.final_norm, cfg.eps), self.lm_head).float()

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        batch, seq = input_ids.shape
        lay = self.seq_layout(batch, seq)
        if lay is not None:
            return self._forward_sp(input_ids, lay)
        cos, sin = rope_tables(seq, cfg.head_dim, cfg.rope_theta, self.device)
        x = torch.nn.functional.embedding(input_ids.reshape(-1), self.embed)  # [T, hidden]
        fuse = self.fuse_residual and self.trace is None
        for i, layer in enumerate(self.layers):
            if fuse:  # the norms inside the qkv / gate_up input quantization, the residual adds in the epilogues
                x = self._attention(layer, x, batch, seq, cos, sin, i, residual=x, norm=(layer.input_norm, cfg.eps))
                gu = layer.gate_up(x, norm=(layer.post_norm, cfg.eps))
            else:
                h = ops.rms_norm(self._t("x", i, x), layer.input_norm, cfg.eps)
                x = self._t("x_mid", i, x + self._attention(layer, h, batch, seq, cos, sin, i))
                gu = self._t("gate_up", i, layer.gate_up(self._t("post_norm", i, ops.rms_norm(x, layer.post_norm,
                                                                                             cfg.eps))))
            if fuse:  # SwiGLU in the down_proj input quantization, the residual add in its epilogue
                x = layer.down(gu, act="swiglu", residual=x)
            else:
                a = self._t("act", i, ops.silu_mul(gu))
                x = x + self._t("down", i, layer.down(a))
        last = self._t("final", len(self.layers), x.view(batch, seq, -1)[:, -1])
        return torch.nn.functional.linear(rms_norm(last, self.final_norm, cfg.eps), self.lm_head).float()


def default_input_ids(batch: int, seq: int, vocab: int, device: torch.device, seed: int = 0) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), generator=g, device=device)


# ---------------------------------------------------------------- Wan2.2 DiT block, heads sharded
@dataclass
class WanBlockConfig:
    """Wan2.2-A14B DiT block shapes; smaller values for tests."""

    dim: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    grid: tuple[int, int, int] = (21, 45, 80)  # latent frames x height x width
    eps: float = 1e-6
    rope_theta: float = 10000.0
    levels: str = "123"
    hisq_seed: int = 17
    seed: int = 0

    @property
    def seq(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    def flops(self) -> dict[str, float]:
        s = self.seq
        attention = 4.0 * self.head_dim * self.heads * s * s
        linear = 2.0 * s * (4 * self.dim * self.dim + 2 * self.dim * self.ffn)
        return {"attention": attention, "linear": linear, "total": attention + linear}


def rope3d_tables(grid: tuple[int, int, int], head_dim: int, theta: float, device: torch.device):
    """fp64 cos/sin ``[F*H*W, head_dim/2]`` of the 3-axis rotary embedding of Wan's DiT
    (Wan's rope_params/rope_apply, which multiply in complex128): the ``head_dim/2``
    complex pairs are split ``[c - 2(c//3), c//3, c//3]`` over (frame, height, width),
    each band with its own ``theta^(-2i/d_band)`` frequencies, and a token at grid
    position (f, h, w) rotates band pairs by (f, h, w) times those frequencies."""
    c = head_dim // 2
    bands = [c - 2 * (c // 3), c // 3, c // 3]
    angles = []
    for axis, (n, pairs) in enumerate(zip(grid, bands)):
        dim = 2 * pairs
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float64) / dim))
        pos = torch.arange(n, device=device, dtype=torch.float64)
        shape = [1, 1, 1, pairs]
        shape[axis] = n
        a = torch.outer(pos, inv).reshape(shape).expand(grid[0], grid[1], grid[2], pairs)
        angles.append(a)
    ang = torch.cat(angles, dim=-1).reshape(-1, c)
    return ang.cos(), ang.sin()


def apply_rope3d(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """torch statement of Wan's rope_apply (the check for ``ops.wan_qk_prep``): ``x [L, H,
    D]`` with channel pairs (2i, 2i+1) as complex numbers, multiplied in fp64 by the fp64
    tables, returned as fp32."""
    xf = x.double().reshape(*x.shape[:-1], -1, 2)
    re, im = xf[..., 0], xf[..., 1]
    c, s = cos.double()[:, None, :], sin.double()[:, None, :]
    out = torch.stack([re * c - im * s, re * s + im * c], dim=-1)
    return out.reshape(x.shape).float()


def wan_qk_norm(t: torch.Tensor, weight: torch.Tensor, heads_total_dim: int, eps: float) -> torch.Tensor:
    """torch statement of WanRMSNorm on the whole q (or k) row ``t [L, dim]`` (the check
    for ``ops.wan_qk_prep``): ``bf16(x * rsqrt(mean(x^2) + eps)) * w``, fp32 out."""
    tf = t.float()
    r = torch.rsqrt(tf.pow(2).sum(-1, keepdim=True) / heads_total_dim + eps)
    return (tf * r).to(torch.bfloat16).float() * weight.float()


class WanBlockTP(nn.Module):
    """One rank of a Wan2.2 DiT block (self-attention + FFN; the text cross-attention and
    the time modulation are not part of the benchmarked block) with every Linear HiF4
    W4A4 and HiF4 QK/PV attention, ``heads / world`` heads on this rank.

    Column-parallel q/k/v and ffn.0 read the LayerNorm outputs with the ``rbhn_r64``
    reader rotation (one HiSQ rotation per norm, 64-channel blocks; shared, so one K1 per
    norm); row-parallel o and ffn.2 use shard-local ``"signs"`` rotations. Wan normalizes
    q and k over all heads (RMSNorm over ``dim``), so the head-sharded form all-gathers
    per-head sums of squares (``[L, 2 heads/world]`` fp32) and K4 adds all heads' sums in
    one fixed order -- the norm, and so the attention operands, are the same bits at
    every TP size; attention itself needs no collective. The glue is one kernel each:
    LayerNorm, the per-head sums, K4 with the norm and the 3-D RoPE in front, GELU.
    """

    def __init__(self, cfg: WanBlockConfig, tp: TPGroup, device: torch.device, index: int = 0) -> None:
        super().__init__()
        self.cfg, self.tp, self.device = cfg, tp, device
        self.trace = None  # trace(stage, 0, tensor) at each stage boundary, as in Qwen3TPPrefill
        self.fuse_residual = True
        self.sequence_parallel = True  # as in Qwen3TPPrefill (off while a trace hook is set)
        self.sp_chunks = 1
        if cfg.heads % tp.world:
            raise ValueError("heads must divide by the TP size")
        d = cfg.head_dim
        self.h_local = cfg.heads // tp.world
        rows = slice(tp.rank * self.h_local * d, (tp.rank + 1) * self.h_local * d)
        f0, fl = tp.shard(cfg.ffn, HIF4_GROUP)
        self.ffn_local = fl
        name = f"blocks.{index}"

        def w(proj: str, n: int, k: int) -> torch.Tensor:
            return random_weight((n, k), _seed(cfg.seed, name, proj), device)

        def b(proj: str, n: int) -> torch.Tensor:
            return random_weight((1, n), _seed(cfg.seed, name, proj, "bias"), device)[0]

        rot1 = column_rotation(f"{name}.norm1", cfg.dim, seed=cfg.hisq_seed, block=64, sharing="linear")
        rot2 = column_rotation(f"{name}.norm2", cfg.dim, seed=cfg.hisq_seed, block=64, sharing="linear")
        wq, wk, wv = (w(f"self_attn.{p}", cfg.dim, cfg.dim)[rows] for p in "qkv")
        bq, bk, bv = (b(f"self_attn.{p}", cfg.dim)[rows] for p in "qkv")
        self.qkv = TPHiF4Linear(torch.cat([wq, wk, wv]), bias=torch.cat([bq, bk, bv]), rotation=rot1,
                                quantize=True, levels=cfg.levels)
        self.o = TPHiF4Linear(w("self_attn.o", cfg.dim, cfg.dim)[:, rows],
                              bias=b("self_attn.o", cfg.dim) if tp.rank == 0 else None, quantize=True,
                              levels=cfg.levels, reduce=tp,
                              rotation=row_rotation(f"{name}.self_attn.o", cfg.dim, tp, seed=cfg.hisq_seed))
        self.ffn0 = TPHiF4Linear(w("ffn.0", cfg.ffn, cfg.dim)[f0:f0 + fl], bias=b("ffn.0", cfg.ffn)[f0:f0 + fl],
                                 rotation=rot2, quantize=True, levels=cfg.levels)
        self.ffn2 = TPHiF4Linear(w("ffn.2", cfg.dim, cfg.ffn)[:, f0:f0 + fl],
                                 bias=b("ffn.2", cfg.dim) if tp.rank == 0 else None, quantize=True,
                                 levels=cfg.levels, reduce=tp,
                                 rotation=row_rotation(f"{name}.ffn.2", cfg.ffn, tp, seed=cfg.hisq_seed))
        self.norm_q = torch.ones(cfg.dim, dtype=torch.float32, device=device)[rows].contiguous()
        self.norm_k = torch.ones(cfg.dim, dtype=torch.float32, device=device)[rows].contiguous()
        self.cos, self.sin = rope3d_tables(cfg.grid, d, cfg.rope_theta, device)

    def seq_layout(self, seq: int) -> SeqLayout | None:
        """The sequence-parallel layout of ``seq`` tokens (None: the replicated path)."""
        if not self.sequence_parallel or self.tp.world == 1 or self.trace is not None:
            return None
        return seq_layout(seq, self.tp, self.sp_chunks)

    def _attend(self, qkv: torch.Tensor, seq: int, tr) -> torch.Tensor:
        """The rank's heads of the self-attention from the qkv output ``[L, 3 hl d]``: Wan's
        q/k RMSNorm over all heads (per-head sums of squares all-gathered), the 3-D RoPE, the
        Hadamard and HiF4 operands (K4), the HiF4 attention (K5); returns ``[L, hl d]``."""
        cfg, d, hl = self.cfg, self.cfg.head_dim, self.h_local
        n = hl * d
        # per-head sums of squares of q and k: [world, L, 2 hl] after the gather
        head_ss = self.tp.all_gather(ops.row_sumsq(qkv[:, :2 * n], segments=2 * hl))
        heads = lambda lo: qkv[:, lo:lo + n].view(1, seq, hl, d).transpose(1, 2)  # noqa: E731
        qd = tr("qd", ops.wan_qk_prep(heads(0), head_ss, self.norm_q, head_offset=0, eps=cfg.eps, cos=self.cos,
                                      sin=self.sin, levels=cfg.levels))
        kd = tr("kd", ops.wan_qk_prep(heads(n), head_ss, self.norm_k, head_offset=hl, eps=cfg.eps, cos=self.cos,
                                      sin=self.sin, levels=cfg.levels))
        vd = tr("vd", ops.qk_prep(heads(2 * n), levels=cfg.levels, rotate=False)[0])
        att = tr("attention", ops.hif4_attention(qd, kd, vd, scale=d ** -0.5, causal=False, p_levels=cfg.levels,
                                                 quantized_normalizer=True))  # [1, L, hl, d]
        return att.view(seq, n)

    @torch.no_grad()
    def forward_shard(self, x_shard: torch.Tensor, lay: SeqLayout) -> torch.Tensor:
        """Sequence-parallel block: ``x_shard`` holds this rank's token rows of the residual
        stream (``lay``, the form consecutive blocks pass on); returns the same rows of the
        block's output. The LayerNorms and the readers' quantization run on the shard, the
        packed codes are all-gathered for the column-parallel q/k/v and ffn.0, and the
        row-parallel o and ffn.2 outputs are reduce-scattered into the shard -- per row the
        arithmetic of the all-reduce path."""
        with self.tp.gemm_sms(x_shard.device):
            return self._forward_shard(x_shard, lay)

    def _forward_shard(self, x_shard: torch.Tensor, lay: SeqLayout) -> torch.Tensor:
        cfg, tp = self.cfg, self.tp
        tr = lambda stage, t: t  # noqa: E731
        qkv = self.qkv.sp_column(x_shard, lay, tp, norm=(None, cfg.eps))
        att = self._attend(qkv, lay.rows, tr)
        x_shard = self.o.sp_row(self.o.quantize_input(att), x_shard, lay, tp)
        f0 = self.ffn0.sp_column(x_shard, lay, tp, norm=(None, cfg.eps))
        return self.ffn2.sp_row(self.ffn2.activate_and_quantize(f0, "gelu_tanh"), x_shard, lay, tp)

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``x [L, dim]`` bf16 (batch 1) -> ``[L, dim]``; with more than one rank the block
        runs sequence-parallel on this rank's rows and the output rows are all-gathered."""
        lay = self.seq_layout(x.shape[0])
        if lay is not None:
            out = self.forward_shard(x[lay.owned(x.device)], lay)
            return sp_gather_rows(self.tp, lay, out)
        cfg = self.cfg
        seq = x.shape[0]
        tr = (lambda stage, t: (self.trace(stage, 0, t), t)[1]) if self.trace is not None else (lambda stage, t: t)
        fuse = self.fuse_residual and self.trace is None  # norms in the readers' K1, residual adds in epilogues
        if fuse:
            qkv = self.qkv(x, norm=(None, cfg.eps))
        else:
            qkv = tr("qkv", self.qkv(tr("norm1", ops.layer_norm(x, cfg.eps))))
        att = self._attend(qkv, seq, tr)
        x = tr("x_mid", self.o(att, residual=x) if fuse else x + tr("o", self.o(att)))
        if fuse:
            f0 = self.ffn0(x, norm=(None, cfg.eps))
        else:
            f0 = tr("ffn0", self.ffn0(tr("norm2", ops.layer_norm(x, cfg.eps))))
        if fuse:  # the GELU in the ffn.2 input quantization, the residual add in its epilogue
            return self.ffn2(f0, act="gelu_tanh", residual=x)
        a = tr("act", ops.gelu_tanh(f0))
        return x + tr("ffn2", self.ffn2(a))
