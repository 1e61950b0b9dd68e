"""Tensor-level entry points over the C ABI (device tensors in, device tensors out).

Each function validates its torch arguments, allocates the outputs with torch
(the library itself never allocates) and launches on the current CUDA stream.
"""

from __future__ import annotations

import os

import torch

from . import _lib

LEVELS = {"123": 123, "12": 12, "13": 13}


def levels_code(levels: str | int) -> int:
    key = str(levels)
    if key not in LEVELS:
        raise ValueError(f"HiF4 levels must be one of {tuple(LEVELS)}, got {levels!r}")
    return LEVELS[key]


def default_levels(kind: str) -> str:
    """The reference's process-wide level variants (``src/faquant/hif4.py:13-43``).

    ``kind`` is ``weight``, ``act`` or one of the attention operands ``q``, ``k``,
    ``p``, ``v``. Read from the same environment variables, at call time.
    """
    weight = os.environ.get("FAQUANT_HIF4_SCALE_LEVELS", "123")
    act = os.environ.get("FAQUANT_HIF4_ACT_SCALE_LEVELS", weight)
    attn = os.environ.get("FAQUANT_HIF4_ATTN_SCALE_LEVELS", act)
    if kind == "weight":
        value = weight
    elif kind == "act":
        value = act
    elif kind in ("q", "k", "p", "v"):
        value = attn
        for entry in filter(None, os.environ.get("FAQUANT_HIF4_ATTN_OPERAND_LEVELS", "").split(",")):
            operand, _, val = entry.partition("=")
            if operand == kind:
                value = val
    else:
        raise ValueError(f"unknown HiF4 operand kind {kind!r}")
    levels_code(value)
    return value


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.FAQ_BF16
    if t.dtype == torch.float32:
        return _lib.FAQ_F32
    raise TypeError(f"unsupported dtype {t.dtype}; the HiF4 kernels take bfloat16 or float32")


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("faquant_b200 operators run on CUDA tensors only (no CPU fallback)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError("all tensors must be on the same CUDA device")
    if device is None:
        raise RuntimeError("no CUDA tensor given")
    return device


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _rows_view(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """``x [..., k]`` as a 2-D row view and its row stride (copies only when needed)."""
    k = x.shape[-1]
    if x.dim() == 2 and x.stride(1) == 1 and x.stride(0) >= k:
        return x, x.stride(0)
    return x.contiguous().reshape(-1, k), k


def hif4_quantize(
    x: torch.Tensor,
    *,
    levels: str | int = "123",
    input_scale: torch.Tensor | None = None,
    signs: torch.Tensor | None = None,
    permutation: torch.Tensor | None = None,
    rot_block: int | None = None,
    want_qdq: bool = True,
    want_codes: bool = False,
) -> tuple[torch.Tensor | None, torch.Tensor | None, torch.Tensor | None]:
    """Rotation (optional) + HiF4 quantization of ``x [..., k]`` along the last axis.

    Returns ``(qdq, codes, meta)``: the dequantized values in ``x.dtype`` (shape of
    ``x``) and the packed codes ``uint8 [rows, k64/2]`` / meta ``int32 [rows, k64/64]``.
    """
    device = _require_cuda(x, input_scale, signs, permutation)
    if x.shape[-1] == 0:
        raise ValueError("HiF4 does not support an empty axis")
    k = x.shape[-1]
    rows, ldx = _rows_view(x)
    n = rows.shape[0]
    k64 = (k + 63) // 64 * 64
    qdq = torch.empty((n, k), dtype=x.dtype, device=device) if want_qdq else None
    codes = torch.empty((n, k64 // 2), dtype=torch.uint8, device=device) if want_codes else None
    meta = torch.empty((n, k64 // 64), dtype=torch.int32, device=device) if want_codes else None
    if input_scale is not None:
        input_scale = input_scale.to(device=device, dtype=x.dtype).contiguous()
        if input_scale.numel() != k:
            raise ValueError("input_scale must have one entry per input channel")
    if signs is not None:
        signs = signs.to(device=device, dtype=torch.int8).contiguous()
        if permutation is not None:
            permutation = permutation.to(device=device, dtype=torch.int64).contiguous()
    block = 0 if rot_block is None else int(rot_block)
    _lib.call(
        "faq_hif4_quantize", rows.data_ptr(), _dtype_code(x), n, k, ldx, _ptr(input_scale), _ptr(signs),
        _ptr(permutation), block, levels_code(levels), _ptr(codes), _ptr(meta), _ptr(qdq), k, _stream(device),
    )
    if qdq is not None:
        qdq = qdq.reshape(x.shape)
    return qdq, codes, meta


ACTIVATIONS = {"swiglu": 1, "gelu_tanh": 2}  # FAQ_ACT_SWIGLU, FAQ_ACT_GELU_TANH


def hif4_quantize_act(
    x: torch.Tensor,
    act: str,
    *,
    levels: str | int = "123",
    input_scale: torch.Tensor | None = None,
    signs: torch.Tensor,
    rot_block: int,
    want_qdq: bool = True,
    want_codes: bool = False,
) -> tuple[torch.Tensor | None, torch.Tensor | None, torch.Tensor | None]:
    """:func:`hif4_quantize` of an activation's output, the activation fused into the load
    (``faq_hif4_quantize_act``): ``act="swiglu"`` takes the gate|up tensor ``x [rows, 2k]``
    and quantizes ``silu_mul(x)``; ``act="gelu_tanh"`` takes ``x [rows, k]`` and quantizes
    ``gelu_tanh(x)`` -- the same outputs as the activation followed by
    :func:`hif4_quantize`, without the activation's tensor. bf16, signs-only rotation
    (block 8..256); returns ``(qdq [rows, k], codes, meta)``."""
    if act not in ACTIVATIONS:
        raise ValueError(f"act must be one of {sorted(ACTIVATIONS)}")
    device = _require_cuda(x, input_scale, signs)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("hif4_quantize_act takes a rank-2 bfloat16 tensor")
    rows = x.shape[0]
    k = x.shape[1] // 2 if act == "swiglu" else x.shape[1]
    if act == "swiglu" and x.shape[1] % 2:
        raise ValueError("the SwiGLU input holds gate and up halves: an even width")
    if x.stride(-1) != 1 or (rows > 1 and x.stride(0) % 8) or x.data_ptr() % 16:
        x = x.contiguous()
    ldx = x.stride(0) if rows > 1 else x.shape[1]
    qdq = torch.empty((rows, k), dtype=torch.bfloat16, device=device) if want_qdq else None
    codes = torch.empty((rows, k // 2), dtype=torch.uint8, device=device) if want_codes else None
    meta = torch.empty((rows, k // 64), dtype=torch.int32, device=device) if want_codes else None
    if input_scale is not None:
        input_scale = input_scale.to(device=device, dtype=torch.bfloat16).contiguous()
    signs = signs.to(device=device, dtype=torch.int8).contiguous()
    _lib.call("faq_hif4_quantize_act", x.data_ptr(), ACTIVATIONS[act], rows, k, ldx, _ptr(input_scale),
              signs.data_ptr(), int(rot_block), levels_code(levels), _ptr(codes), _ptr(meta), _ptr(qdq), k,
              _stream(device))
    return qdq, codes, meta


def rms_norm_quantize_supported(k: int, rot_block: int | None) -> bool:
    """Whether :func:`hif4_quantize_rms_norm` takes a row of ``k`` channels rotated in
    blocks of ``rot_block`` (the K1 v4 shapes: k % 1024 == 0, k <= 16384, 32..1024)."""
    return (rot_block is not None and k % 1024 == 0 and k <= 16384 and 32 <= rot_block <= 1024
            and rot_block & (rot_block - 1) == 0)


def hif4_quantize_rms_norm(
    x: torch.Tensor,
    norm_weight: torch.Tensor | None,
    eps: float,
    *,
    levels: str | int = "123",
    input_scale: torch.Tensor | None = None,
    signs: torch.Tensor,
    permutation: torch.Tensor | None = None,
    rot_block: int,
    want_meta: bool = False,
    want_qdq: bool = True,
    codes_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """:func:`hif4_quantize` of ``rms_norm(x, norm_weight, eps)`` in one pass
    (``faq_hif4_quantize_rms_norm``): the same bits as :func:`rms_norm` followed by
    :func:`hif4_quantize`, without the normalized tensor in memory. bf16 ``x [rows, k]``
    with ``rms_norm_quantize_supported(k, rot_block)``; returns ``(qdq, meta)``
    (``qdq`` None with ``want_qdq=False``). ``codes_out`` (``uint8 [rows, k/2]``,
    contiguous) receives the packed codes as well. ``norm_weight=None`` takes the
    affine-free LayerNorm instead (``faq_hif4_quantize_layer_norm``, the bits of
    :func:`layer_norm` then :func:`hif4_quantize`)."""
    device = _require_cuda(x, norm_weight, input_scale, signs, permutation)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("hif4_quantize_rms_norm takes a rank-2 bfloat16 tensor")
    rows, k = x.shape
    if x.stride(-1) != 1 or (rows > 1 and x.stride(0) % 8) or x.data_ptr() % 16:
        x = x.contiguous()
    ldx = x.stride(0) if rows > 1 else k
    qdq = torch.empty((rows, k), dtype=torch.bfloat16, device=device) if want_qdq else None
    meta = torch.empty((rows, k // 64), dtype=torch.int32, device=device) if want_meta else None
    if codes_out is not None:
        if (codes_out.dtype != torch.uint8 or tuple(codes_out.shape) != (rows, k // 2)
                or not codes_out.is_contiguous() or codes_out.device != device):
            raise ValueError("codes_out must be a contiguous uint8 [rows, k/2] tensor on x's device")
    elif not want_qdq:
        raise ValueError("nothing to write: want_qdq=False without codes_out")
    if input_scale is not None:
        input_scale = input_scale.to(device=device, dtype=torch.bfloat16).contiguous()
    signs = signs.to(device=device, dtype=torch.int8).contiguous()
    if permutation is not None:
        permutation = permutation.to(device=device, dtype=torch.int64).contiguous()
    tail = (_ptr(input_scale), signs.data_ptr(), _ptr(permutation), int(rot_block), levels_code(levels),
            _ptr(codes_out), _ptr(meta), _ptr(qdq), k, _stream(device))
    if norm_weight is None:
        _lib.call("faq_hif4_quantize_layer_norm", x.data_ptr(), rows, k, ldx, float(eps), *tail)
    else:
        norm_weight = norm_weight.to(device=device, dtype=torch.bfloat16).contiguous()
        _lib.call("faq_hif4_quantize_rms_norm", x.data_ptr(), rows, k, ldx, norm_weight.data_ptr(), float(eps), *tail)
    return qdq, meta


def hif4_dequantize(codes: torch.Tensor, meta: torch.Tensor, k: int, dtype: torch.dtype = torch.bfloat16,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed HiF4 ``codes [rows, k64/2]`` / ``meta [rows, k64/64]`` -> values ``[rows, k]``
    (into ``out`` when given: any row stride, unit column stride)."""
    device = _require_cuda(codes, meta, out)
    rows = codes.shape[0]
    if out is None:
        out = torch.empty((rows, k), dtype=dtype, device=device)
    elif out.shape != (rows, k) or out.stride(-1) != 1 or out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out must be a bf16/fp32 [rows, k] tensor with unit column stride")
    ldo = out.stride(0) if rows > 1 else k
    _lib.call("faq_hif4_dequantize", codes.contiguous().data_ptr(), meta.contiguous().data_ptr(), rows, k,
              out.data_ptr(), _dtype_code(out), ldo, _stream(device))
    return out


def hif4_pack_weight(
    weight: torch.Tensor,
    *,
    levels: str | int = "123",
    scale: torch.Tensor | None = None,
    lv2: torch.Tensor | None = None,
    lv3: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Pack an ``[n, k]`` HiF4-grid weight; returns ``(codes, meta, mismatches)``."""
    device = _require_cuda(weight)
    n, k = weight.shape
    k64 = (k + 63) // 64 * 64
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    codes = torch.empty((n, k64 // 2), dtype=torch.uint8, device=device)
    meta = torch.empty((n, k64 // 64), dtype=torch.int32, device=device)
    counter = torch.zeros(1, dtype=torch.int64, device=device)
    if scale is not None:
        scale = scale.to(device=device, dtype=torch.float32).reshape(n, k // 64).contiguous()
        lv2 = lv2.to(device=device, dtype=torch.int8).reshape(n, k // 64, 8).contiguous()
        lv3 = lv3.to(device=device, dtype=torch.int8).reshape(n, k // 64, 16).contiguous()
    _lib.call("faq_hif4_pack_weight", w.data_ptr(), _dtype_code(w), n, k, w.stride(0), _ptr(scale), _ptr(lv2),
              _ptr(lv3), levels_code(levels), codes.data_ptr(), meta.data_ptr(), counter.data_ptr(), _stream(device))
    return codes, meta, int(counter.item())


def set_gemm_sm_target(sms: int) -> None:
    """Size the persistent GEMMs' grids for ``sms`` SMs from the next launch on (0: every
    SM; ``faq_set_gemm_sm_target``): leaves SMs free for collectives that run beside them."""
    _lib.call("faq_set_gemm_sm_target", int(sms))


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None,
              out: torch.Tensor | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``a [m, k] @ b [n, k]^T (+ bias)`` in bf16 with fp32 accumulation (tcgen05); with
    ``residual [m, n]`` (bf16) the result is ``residual + that`` with the eager bf16 add's
    rounding (the product rounded to bf16 first), added in the GEMM's epilogue."""
    device = _require_cuda(a, b, bias, residual)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm_bf16 takes bfloat16 operands")
    if a.stride(-1) != 1:
        a = a.contiguous()
    if b.stride(-1) != 1:
        b = b.contiguous()
    m, k = a.shape
    n = b.shape[0]
    if b.shape[1] != k:
        raise ValueError("inner dimensions differ")
    lda = a.stride(0) if m > 1 else k
    ldb = b.stride(0) if n > 1 else k
    if k % 8 or lda % 8 or ldb % 8 or a.data_ptr() % 16 or b.data_ptr() % 16:
        # TMA wants 16-byte aligned rows: pad k with zeros, which adds nothing to the sums
        k8 = (k + 7) // 8 * 8
        a = torch.nn.functional.pad(a, (0, k8 - k))
        b = torch.nn.functional.pad(b, (0, k8 - k))
        k, lda, ldb = k8, k8, k8
    if bias is not None:
        bias = bias.to(device=device, dtype=torch.bfloat16).contiguous()
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=device)
    if residual is None:
        _lib.call("faq_gemm_bf16_tn", a.data_ptr(), lda, b.data_ptr(), ldb, m, n, k, _ptr(bias), out.data_ptr(),
                  out.stride(0) if m > 1 else n, _stream(device))
        return out
    if residual.dtype != torch.bfloat16 or residual.shape != (m, n):
        raise ValueError("residual must be bfloat16 [m, n]")
    if residual.stride(-1) != 1:
        residual = residual.contiguous()
    _lib.call("faq_gemm_bf16_tn_residual", a.data_ptr(), lda, b.data_ptr(), ldb, m, n, k, _ptr(bias),
              residual.data_ptr(), residual.stride(0) if m > 1 else n, out.data_ptr(),
              out.stride(0) if m > 1 else n, _stream(device))
    return out


def w4a4_gemm(a: torch.Tensor | tuple[torch.Tensor, torch.Tensor], b_codes: torch.Tensor, b_meta: torch.Tensor,
              bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
              residual: torch.Tensor | None = None) -> torch.Tensor:
    """The W4A4 GEMM on a packed HiF4 weight ``(b_codes uint8 [n, k/2], b_meta int32
    [n, k/64])``: ``deq(a) @ deq(b)^T (+ bias) (+ residual)`` in bf16, bit-identical to
    ``gemm_bf16`` on the dequantized operands. ``a`` is the activation's packed form
    ``(codes, meta)`` (``hif4_quantize(..., want_codes=True)``) or its bf16 QDQ ``[m, k]``;
    a bf16 ``a`` of at most 16 rows runs the small-row kernel, whose sums run in another
    order (the same values up to fp32 rounding of the accumulation). ``k`` must be a
    multiple of 256 (``NotImplementedError`` otherwise)."""
    device = _require_cuda(b_codes, b_meta, bias, residual)
    if b_codes.dtype != torch.uint8 or b_meta.dtype not in (torch.int32, torch.uint32):
        raise TypeError("packed weight: codes uint8 [n, k/2], meta int32 [n, k/64]")
    n = b_codes.shape[0]
    k = b_codes.shape[1] * 2
    if b_meta.shape != (n, k // 64):
        raise ValueError("packed weight: meta must be [n, k/64]")
    b_codes, b_meta = b_codes.contiguous(), b_meta.contiguous()
    packed_a = isinstance(a, tuple)
    if packed_a:
        a_codes, a_meta = (t.contiguous() for t in a)
        _require_cuda(a_codes, a_meta)
        m = a_codes.shape[0]
        if a_codes.dtype != torch.uint8 or a_codes.shape[1] * 2 != k or a_meta.shape != (m, k // 64):
            raise ValueError("packed activation: codes uint8 [m, k/2] and meta [m, k/64] with the weight's k")
    else:
        _require_cuda(a)
        if a.dtype != torch.bfloat16 or a.shape[-1] != k:
            raise ValueError("the QDQ activation must be bfloat16 [m, k] with the weight's k")
        if a.stride(-1) != 1 or a.stride(0) % 8 or a.data_ptr() % 16:
            a = a.contiguous()
        m = a.shape[0]
    if bias is not None:
        bias = bias.to(device=device, dtype=torch.bfloat16).contiguous()
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=device)
    ldr = 0
    if residual is not None:
        if residual.dtype != torch.bfloat16 or residual.shape != (m, n):
            raise ValueError("residual must be bfloat16 [m, n]")
        if residual.stride(-1) != 1:
            residual = residual.contiguous()
        ldr = residual.stride(0) if m > 1 else n
    ldy = out.stride(0) if m > 1 else n
    if packed_a:
        _lib.call("faq_w4a4_gemm", a_codes.data_ptr(), a_meta.data_ptr(), b_codes.data_ptr(), b_meta.data_ptr(),
                  m, n, k, _ptr(bias), _ptr(residual), ldr, out.data_ptr(), ldy, _stream(device))
    else:
        lda = a.stride(0) if m > 1 else k
        _lib.call("faq_w4a4_gemm_qdq_a", a.data_ptr(), lda, b_codes.data_ptr(), b_meta.data_ptr(), m, n, k,
                  _ptr(bias), _ptr(residual), ldr, out.data_ptr(), ldy, _stream(device))
    return out


def selftest_wait_timeout(limit_ns: int) -> None:
    device = torch.device("cuda", torch.cuda.current_device())
    _lib.call("faq_selftest_wait_timeout", int(limit_ns), _stream(device))


def qk_prep(
    x: torch.Tensor,
    *,
    levels: str | int | None = "123",
    rotate: bool = True,
    smooth_scale: torch.Tensor | None = None,
    smooth_mode: str | None = None,
    key_offset: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    want_codes: bool = False,
) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """Attention operand preparation of ``x [B, H, S, D]`` (any strides, D contiguous).

    ``smooth_mode`` is ``"mul"`` (Q), ``"div"`` (K) or None; ``smooth_scale`` is
    ``[D]`` or ``[H, D]``; ``key_offset`` is ``[H, D]`` (K only). Returns the bf16
    operand ``[B, H, S, D]`` (``out`` if given) and optional packed codes/meta.
    """
    device = _require_cuda(x, smooth_scale, key_offset)
    if x.dim() != 4:
        raise ValueError("qk_prep expects [batch, heads, seq, head_dim]")
    b, h, s, d = x.shape
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=device)
    mode = {None: 0, "mul": 1, "div": 2}[smooth_mode]
    head_stride = 0
    if smooth_scale is not None:
        smooth_scale = smooth_scale.to(device=device, dtype=torch.float32).contiguous()
        head_stride = d if smooth_scale.dim() == 2 else 0
    if key_offset is not None:
        key_offset = key_offset.to(device=device, dtype=torch.float32).reshape(h, d).contiguous()
    lv = 0 if levels is None else levels_code(levels)
    codes = meta = None
    if want_codes and lv:
        codes = torch.empty((b * h * s, d // 2), dtype=torch.uint8, device=device)
        meta = torch.empty((b * h * s, d // 64), dtype=torch.int32, device=device)
    _lib.call("faq_qk_prep", x.data_ptr(), _dtype_code(x), b, h, s, d, x.stride(0), x.stride(1), x.stride(2),
              _ptr(key_offset), _ptr(smooth_scale), head_stride, mode, int(rotate), lv, out.data_ptr(),
              out.stride(0), out.stride(1), out.stride(2), _ptr(codes), _ptr(meta), _stream(device))
    return out, codes, meta


def qk_norm_rope_prep(
    x: torch.Tensor,
    *,
    norm_weight: torch.Tensor | None,
    eps: float = 1e-6,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    levels: str | int | None = "123",
    rotate: bool = True,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Qwen3 attention operand in one pass: per-head RMSNorm (``norm_weight [D]`` bf16),
    RoPE (bf16 ``cos``/``sin`` ``[S, D]``, position = sequence index), Hadamard over D,
    bf16, HiF4. ``x [B, H, S, D]`` bf16, any strides with D contiguous."""
    device = _require_cuda(x, norm_weight, cos, sin)
    if x.dim() != 4 or x.dtype != torch.bfloat16:
        raise ValueError("qk_norm_rope_prep expects bf16 [batch, heads, seq, head_dim]")
    b, h, s, d = x.shape
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=device)
    if norm_weight is not None:
        norm_weight = norm_weight.to(device=device, dtype=torch.bfloat16).contiguous()
    rope_ld = 0
    if cos is not None:
        cos = cos.to(device=device, dtype=torch.bfloat16).contiguous()
        sin = sin.to(device=device, dtype=torch.bfloat16).contiguous()
        if cos.shape[0] < s or cos.shape[-1] != d:
            raise ValueError("cos/sin must be [>= seq, head_dim]")
        rope_ld = cos.stride(0)
    lv = 0 if levels is None else levels_code(levels)
    _lib.call("faq_qk_norm_rope_prep", x.data_ptr(), _dtype_code(x), b, h, s, d, x.stride(0), x.stride(1),
              x.stride(2), _ptr(norm_weight), float(eps), _ptr(cos), _ptr(sin), rope_ld, None, None, 0, 0,
              int(rotate), lv, out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), None, None,
              _stream(device))
    return out


def wan_qk_prep(
    x: torch.Tensor,
    head_sumsq: torch.Tensor,
    norm_weight: torch.Tensor,
    *,
    head_offset: int = 0,
    eps: float = 1e-6,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    smooth_scale: torch.Tensor | None = None,
    smooth_mode: str | None = None,
    levels: str | int | None = "123",
    rotate: bool = True,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Wan2.2 self-attention operand in one pass: WanRMSNorm over each token's whole row
    of all heads, the 3-D RoPE (fp64 ``cos``/``sin`` ``[S, D/2]``), optional Smooth-QK,
    Hadamard over D, bf16, HiF4. ``x [B, H, S, D]`` bf16, any strides with D contiguous.

    ``head_sumsq [ranks, B*S, C]`` fp32 holds per-head sums of squares (``row_sumsq``
    with one segment per head; ``ranks`` > 1 when gathered from a head-sharded layer):
    this tensor's heads of rank r are columns ``head_offset .. head_offset + H`` of
    block r, so the norm runs over ``ranks * H`` heads. ``norm_weight [H, D]`` or
    ``[H*D]`` is this shard's weight."""
    device = _require_cuda(x, head_sumsq, norm_weight, cos, sin, smooth_scale)
    if x.dim() != 4 or x.dtype != torch.bfloat16:
        raise ValueError("wan_qk_prep expects bf16 [batch, heads, seq, head_dim]")
    b, h, s, d = x.shape
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=device)
    if head_sumsq.dtype != torch.float32 or head_sumsq.dim() != 3 or not head_sumsq.is_contiguous():
        raise TypeError("head_sumsq must be a contiguous fp32 [ranks, batch * seq, columns] tensor")
    ranks, tokens, cols = head_sumsq.shape
    if tokens != b * s or head_offset < 0 or head_offset + h > cols:
        raise ValueError("head_sumsq does not cover these heads and tokens")
    norm_weight = norm_weight.to(device=device, dtype=torch.float32).reshape(h, d).contiguous()
    if cos is not None:
        cos = cos.to(device=device, dtype=torch.float64).contiguous()
        sin = sin.to(device=device, dtype=torch.float64).contiguous()
        if cos.shape != (s, d // 2) or sin.shape != (s, d // 2):
            raise ValueError("cos/sin must be [seq, head_dim / 2]")
    mode = {None: 0, "mul": 1, "div": 2}[smooth_mode]
    head_stride = 0
    if smooth_scale is not None:
        smooth_scale = smooth_scale.to(device=device, dtype=torch.float32).contiguous()
        head_stride = d if smooth_scale.dim() == 2 else 0
    lv = 0 if levels is None else levels_code(levels)
    _lib.call("faq_wan_qk_prep", x.data_ptr(), b, h, s, d, x.stride(0), x.stride(1), x.stride(2),
              head_sumsq.data_ptr() + 4 * head_offset, ranks * h, h, cols, tokens * cols, norm_weight.data_ptr(),
              float(eps), _ptr(cos), _ptr(sin),
              _ptr(smooth_scale), head_stride, mode, int(rotate), lv, out.data_ptr(), out.stride(0), out.stride(1),
              out.stride(2), _stream(device))
    return out


def row_sumsq(x: torch.Tensor, segments: int = 1, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 ``[rows, segments]`` sums of squares of the ``segments`` equal column blocks
    of bf16 ``x [rows, cols]`` (a column slice of a wider tensor is fine)."""
    device = _require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("row_sumsq takes a bf16 [rows, cols] tensor with contiguous rows")
    rows, cols = x.shape
    if cols % segments:
        raise ValueError("cols must divide into the segments")
    if out is None:
        out = torch.empty((rows, segments), dtype=torch.float32, device=device)
    _lib.call("faq_row_sumsq", x.data_ptr(), rows, segments, cols // segments, x.stride(0) if rows > 1 else cols,
              out.data_ptr(), _stream(device))
    return out


def layer_norm(x: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm without affine of bf16 ``x [..., k]`` (fp32 statistics), one pass."""
    device = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("layer_norm takes bfloat16")
    rows, ldx = _rows_view(x)
    k = x.shape[-1]
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=device)
    _lib.call("faq_layer_norm", rows.data_ptr(), rows.shape[0], k, ldx, float(eps), out.data_ptr(), k,
              _stream(device))
    return out


def gelu_tanh(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """GELU (tanh approximation) of a bf16 ``[rows, cols]`` tensor, one pass."""
    device = _require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("gelu_tanh takes a bf16 [rows, cols] tensor with contiguous rows")
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=device)
    _lib.call("faq_gelu_tanh", x.data_ptr(), rows, cols, x.stride(0) if rows > 1 else cols, out.data_ptr(),
              out.stride(0) if rows > 1 else cols, _stream(device))
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3RMSNorm of bf16 ``x [..., k]`` in one pass."""
    device = _require_cuda(x, weight)
    if x.dtype != torch.bfloat16:
        raise TypeError("rms_norm takes bfloat16")
    rows, ldx = _rows_view(x)
    k = x.shape[-1]
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=device)
    weight = weight.to(device=device, dtype=torch.bfloat16).contiguous()
    _lib.call("faq_rms_norm", rows.data_ptr(), rows.shape[0], k, ldx, weight.data_ptr(), float(eps), out.data_ptr(),
              k, _stream(device))
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up`` of a bf16 ``[rows, 2f]`` gate|up tensor, one pass."""
    device = _require_cuda(gate_up)
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or gate_up.stride(1) != 1:
        raise TypeError("silu_mul takes a bf16 [rows, 2f] tensor with contiguous rows")
    rows, two_f = gate_up.shape
    f = two_f // 2
    if out is None:
        out = torch.empty((rows, f), dtype=torch.bfloat16, device=device)
    _lib.call("faq_silu_mul", gate_up.data_ptr(), rows, f, gate_up.stride(0), out.data_ptr(), out.stride(0),
              _stream(device))
    return out


def hif4_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float | None = None,
    causal: bool = True,
    p_levels: str | int | None = "123",
    quantized_normalizer: bool = True,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """HiF4 QK/PV attention of pre-quantized bf16 operands.

    ``q [B, Hq, Sq, 128]``, ``k/v [B, Hkv, Sk, 128]`` (any strides with the head dim
    contiguous); returns ``[B, Sq, Hq, 128]`` bf16 (``out`` if given).
    """
    device = _require_cuda(q, k, v)
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.dim() != 4:
            raise TypeError("hif4_attention takes rank-4 bfloat16 Q/K/V")
    b, hq, sq, d = q.shape
    _, hkv, sk, _ = k.shape
    if v.shape != k.shape:
        raise ValueError("K and V shapes differ")

    def fix(t: torch.Tensor) -> torch.Tensor:
        ok = t.stride(-1) == 1 and all(st % 8 == 0 for st in t.stride()[:-1]) and t.data_ptr() % 16 == 0
        return t if ok else t.contiguous()

    q, k, v = fix(q), fix(k), fix(v)
    if out is None:
        out = torch.empty((b, sq, hq, d), dtype=torch.bfloat16, device=device)
    scale = float(scale if scale is not None else d**-0.5)
    lv = 0 if p_levels is None else levels_code(p_levels)
    _lib.call("faq_hif4_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), b, hq, hkv, sq, sk, d,
              q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
              v.stride(0), v.stride(1), v.stride(2), scale, int(causal), lv, int(quantized_normalizer),
              out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), _stream(device))
    return out


def hif4_decode_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float | None = None,
    p_levels: str | int | None = "123",
    quantized_normalizer: bool = True,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode-step HiF4 attention: ``q [B, Hq, Sq, 128]`` (the last Sq positions, Sq small)
    against ``k/v [B, Hkv, Sk, 128]`` (the whole cache), pre-quantized bf16 operands;
    returns ``[B, Sq, Hq, 128]``. Same semantics as :func:`hif4_attention` with causal
    masking; the keys are split over the GPU (exact running max per tile)."""
    device = _require_cuda(q, k, v)
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.dim() != 4:
            raise TypeError("hif4_decode_attention takes rank-4 bfloat16 Q/K/V")
    b, hq, sq, d = q.shape
    _, hkv, sk, _ = k.shape
    if v.shape != k.shape:
        raise ValueError("K and V shapes differ")
    def fix(t: torch.Tensor) -> torch.Tensor:
        ok = t.stride(-1) == 1 and all(st % 8 == 0 for st in t.stride()[:-1]) and t.data_ptr() % 16 == 0
        return t if ok else t.contiguous()

    q, k, v = fix(q), fix(k), fix(v)
    need = int(_lib.load().faq_hif4_decode_workspace_bytes(b, hq, hkv, sq, sk, d))
    if need == 0:
        raise ValueError("unsupported decode shape")
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    if out is None:
        out = torch.empty((b, sq, hq, d), dtype=torch.bfloat16, device=device)
    scale = float(scale if scale is not None else d**-0.5)
    lv = 0 if p_levels is None else levels_code(p_levels)
    _lib.call("faq_hif4_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), b, hq, hkv, sq, sk, d,
              q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
              v.stride(2), scale, lv, int(quantized_normalizer), out.data_ptr(), out.stride(0), out.stride(1),
              out.stride(2), workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream(device))
    return out
