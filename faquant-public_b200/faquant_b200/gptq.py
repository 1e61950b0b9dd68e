"""GPTQ with HiF4 grids on the GPU: the drop-in for ``faquant.gptq.GPTQ``.

Reference: ``src/faquant/gptq.py`` -- ``GPTQ`` (:123), ``add_batch`` (:164-172),
``_damped_inverse_cholesky`` (:174-195), ``_quantize_block_diagonal`` (:197-298) and
``quantize`` (:324-593), for the configuration the deployed recipes use
(``GPTQ_SETTINGS``, ``workflows/wan22_gptq.py:58``: HiF4, 4 bits, groups of 64, symmetric,
block 128; full Hessian, or the block-diagonal form with 64-column Hessian blocks).

The work is split as the algorithm splits it:
- the Hessian ``H += X^T X`` and the lazy update of later columns
  ``W[:, stop:] -= E @ H^-1[block, stop:]`` are plain fp32 GEMMs (torch on the GPU);
- the damped inverse Cholesky factor is torch.linalg on the GPU, the reference's retry
  chain unchanged;
- the column loop -- HiF4 fit at each group start from the current values, quantization,
  error, rank-1 update -- is this library's ``faq_gptq_hif4_block`` kernel, one warp per
  weight row, with the reference's single fp32 roundings.

The arithmetic is the reference's; the fp32 GEMMs and the Cholesky factorization sum in
another order than the CPU libraries, so values can differ in last bits before a
quantization step -- the grid and metadata are compared with the reference's CPU solver
in ``tests/test_gpu_gptq.py``. Knobs outside the deployed recipe (integer formats, scale
search, in-group act-order, latent-master capture) raise ``NotImplementedError``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

from . import _lib, ops

HIF4_BLOCK_SIZE = 64


@dataclass
class CompactHiF4Parameters:
    """The reference's ``CompactHiF4Parameters`` (hif4.py:67-79), this solver's shapes:
    scale/reciprocal ``[N, K/64, 1, 1, 1]``, lv2 ``[N, K/64, 8, 1, 1]``, lv3
    ``[N, K/64, 8, 2, 1]`` (the shapes GPTQ.quantize captures, gptq.py:407-423)."""

    scale: torch.Tensor
    reciprocal: torch.Tensor
    scale_lv2_exponent: torch.Tensor
    scale_lv3_exponent: torch.Tensor


@dataclass(frozen=True)
class GPTQStats:
    samples: int
    mean_loss: float
    damp_multiplier: float
    scale_step_counts: dict[int, int] = field(default_factory=dict)


class GPTQ:
    """Layer-local GPTQ with HiF4 grids; the layer must live on a CUDA device."""

    def __init__(self, layer: nn.Linear, *, hessian_block_size: int | None = None) -> None:
        if not isinstance(layer, nn.Linear):
            raise TypeError("GPTQ expects nn.Linear")
        if not layer.weight.is_cuda:
            raise RuntimeError("faquant_b200.gptq.GPTQ solves on the GPU: move the layer to CUDA first")
        self.layer = layer
        self.columns = layer.in_features
        self.hessian_block_size = hessian_block_size
        if hessian_block_size is None:
            shape = (self.columns, self.columns)
        else:
            if hessian_block_size <= 0 or self.columns % hessian_block_size:
                raise ValueError("hessian_block_size must be a positive divisor of in_features")
            shape = (self.columns // hessian_block_size, hessian_block_size, hessian_block_size)
        self.hessian = torch.zeros(shape, device=layer.weight.device, dtype=torch.float32)
        self.samples = 0
        self.weight_override: torch.Tensor | None = None

    def set_weight_override(self, weight: torch.Tensor) -> None:
        if tuple(weight.shape) != tuple(self.layer.weight.shape):
            raise ValueError("GPTQ weight override shape mismatch")
        if not torch.isfinite(weight).all():
            raise ValueError("GPTQ weight override must be finite")
        self.weight_override = weight.detach().float()

    def _source_weight(self) -> torch.Tensor:
        src = self.weight_override if self.weight_override is not None else self.layer.weight.detach()
        return src.float().to(self.layer.weight.device).clone()

    @torch.inference_mode()
    def add_batch(self, inputs: torch.Tensor) -> None:
        """``H += X^T X`` over the calibration rows (gptq.py:164-172), fp32 on the GPU."""
        x = inputs.reshape(-1, inputs.shape[-1]).to(self.hessian.device).float()
        if self.hessian_block_size is None:
            self.hessian.add_(x.T @ x)
        else:
            grouped = x.reshape(x.shape[0], -1, self.hessian_block_size)
            self.hessian.add_(torch.einsum("ngi,ngj->gij", grouped, grouped))
        self.samples += x.shape[0]

    @staticmethod
    def _damped_inverse_cholesky(hessian: torch.Tensor, base_damp: torch.Tensor) -> tuple[torch.Tensor, float]:
        """The upper Cholesky factor of the damped inverse, retrying with 10x more damping
        (gptq.py:174-195)."""
        diagonal = torch.arange(hessian.shape[-1], device=hessian.device)
        for multiplier in (1.0, 10.0, 100.0, 1000.0):
            candidate = hessian.clone()
            candidate[..., diagonal, diagonal] += base_damp[..., None] * multiplier
            factor, info = torch.linalg.cholesky_ex(candidate)
            if torch.any(info):
                continue
            inverse = torch.cholesky_inverse(factor)
            inverse = (inverse + inverse.transpose(-1, -2)) * 0.5
            inverse_factor, inverse_info = torch.linalg.cholesky_ex(inverse, upper=True)
            if not torch.any(inverse_info) and torch.isfinite(inverse_factor).all():
                return inverse_factor.contiguous(), multiplier
        raise RuntimeError("GPTQ Hessian or its inverse is not positive definite after damping")

    def _block(self, w: torch.Tensor, cols: int, nblocks: int, hinv: torch.Tensor, hinv_stride: int,
               q: torch.Tensor, err: torch.Tensor, meta: tuple[torch.Tensor, ...], group0: int, levels: str) -> None:
        scale, rec, lv2, lv3 = meta
        rows = w.shape[0]
        gpr = scale.shape[1]
        dev = w.device
        _lib.call("faq_gptq_hif4_block", w.data_ptr(), w.stride(0), rows, cols, nblocks, hinv.data_ptr(),
                  hinv.stride(-2), hinv_stride, ops.levels_code(levels), q.data_ptr(), q.stride(0),
                  err.data_ptr(), err.stride(0), scale[:, group0:].data_ptr(), rec[:, group0:].data_ptr(),
                  lv2[:, group0:].data_ptr(), lv3[:, group0:].data_ptr(), gpr, ops._stream(dev))

    @torch.inference_mode()
    def quantize(
        self,
        *,
        quant_format: str = "int",
        bits: int = 4,
        group_size: int = 128,
        symmetric: bool = True,
        damp: float = 0.01,
        block_size: int = 128,
        capture_hif4_metadata: bool = False,
        capture_latent_master: bool = False,
        scale_search_steps: tuple[int, ...] | None = None,
        act_order_within_group: bool = False,
    ) -> GPTQStats:
        """Quantize the layer's weight in place (gptq.py:324-593); the argument rules are the
        reference's. With ``capture_hif4_metadata`` the compact metadata is stored in
        ``layer.faquant_hif4_qat_parameters``."""
        if self.samples == 0:
            raise RuntimeError("GPTQ requires calibration samples")
        if block_size <= 0:
            raise ValueError("GPTQ block_size must be positive")
        if quant_format not in ("int", "hif4"):
            raise ValueError(f"unsupported quant_format={quant_format!r}")
        if quant_format != "hif4":
            raise NotImplementedError("faquant_b200 solves GPTQ with HiF4 grids only")
        if group_size == -1:
            group_size = self.columns
        if bits != 4 or not symmetric:
            raise ValueError("HiF4 GPTQ requires 4-bit sign-magnitude quantization")
        if group_size != HIF4_BLOCK_SIZE:
            raise ValueError("HiF4 GPTQ requires group_size=64")
        if block_size % HIF4_BLOCK_SIZE:
            raise ValueError("HiF4 GPTQ block_size must be a multiple of 64")
        if capture_latent_master and not capture_hif4_metadata:
            raise ValueError("latent-master capture requires HiF4 metadata")
        if self.columns % group_size:
            raise ValueError("GPTQ group_size must divide layer.in_features")
        if scale_search_steps is not None or act_order_within_group or capture_latent_master:
            raise NotImplementedError("scale search, in-group act-order and latent-master capture are not "
                                      "part of the deployed recipe and are not implemented on the GPU")
        if block_size not in (64, 128):
            raise NotImplementedError("the GPU solver's column loop takes blocks of 64 or 128 columns")
        levels = ops.default_levels("weight")
        weight = self._source_weight()
        original = weight.clone()
        rows, cols = weight.shape
        groups = cols // HIF4_BLOCK_SIZE
        dev = weight.device
        scale = torch.empty((rows, groups), device=dev, dtype=torch.float32)
        rec = torch.empty_like(scale)
        lv2 = torch.empty((rows, groups, 8), device=dev, dtype=torch.int8)
        lv3 = torch.empty((rows, groups, 16), device=dev, dtype=torch.int8)
        quantized = torch.empty_like(weight)
        errors = torch.empty_like(weight)
        hessian = self.hessian / self.samples
        if self.hessian_block_size is not None:
            # block-diagonal form (gptq.py:197-298): independent 64-column groups, each
            # with its own H^-1 block and its HiF4 fit from the initial values
            if self.hessian_block_size != group_size:
                raise ValueError("block-diagonal GPTQ requires Hessian blocks to match weight groups")
            dead = torch.diagonal(hessian, dim1=-2, dim2=-1) == 0
            diag = torch.arange(group_size, device=dev)
            hessian[:, diag, diag] = torch.where(dead, torch.ones_like(hessian[:, diag, diag]),
                                                 hessian[:, diag, diag])
            weight.view(rows, groups, group_size).masked_fill_(dead.unsqueeze(0), 0)
            base_damp = damp * torch.diagonal(hessian, dim1=-2, dim2=-1).mean(dim=-1).clamp_min(1e-8)
            hinv, multiplier = self._damped_inverse_cholesky(hessian, base_damp)
            self._block(weight, group_size, groups, hinv, group_size * group_size, quantized, errors,
                        (scale, rec, lv2, lv3), 0, levels)
        else:
            dead = torch.diag(hessian) == 0
            hessian[dead, dead] = 1
            weight[:, dead] = 0
            base_damp = damp * torch.diag(hessian).mean().clamp_min(1e-8)
            hinv, multiplier = self._damped_inverse_cholesky(hessian, base_damp)
            for start in range(0, cols, block_size):
                stop = min(start + block_size, cols)
                width = stop - start
                self._block(weight[:, start:stop], width, 1, hinv[start:stop, start:stop], 0,
                            quantized[:, start:stop], errors[:, start:stop], (scale, rec, lv2, lv3),
                            start // HIF4_BLOCK_SIZE, levels)
                if stop < cols:
                    weight[:, stop:] -= errors[:, start:stop] @ hinv[start:stop, stop:]
        self.layer.weight.data.copy_(quantized.to(self.layer.weight.dtype))
        if capture_hif4_metadata:
            self.layer.faquant_hif4_qat_parameters = CompactHiF4Parameters(
                scale=scale.reshape(rows, groups, 1, 1, 1),
                reciprocal=rec.reshape(rows, groups, 1, 1, 1),
                scale_lv2_exponent=lv2.reshape(rows, groups, 8, 1, 1),
                scale_lv3_exponent=lv3.reshape(rows, groups, 8, 2, 1),
            )
        mean_loss = (original - quantized).square().mean().item()
        self.hessian = torch.empty(0, device=dev)
        return GPTQStats(samples=self.samples, mean_loss=mean_loss, damp_multiplier=multiplier)
