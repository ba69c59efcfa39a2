"""Drop-in for the reference's `cuda_decode_gemv` module (decode GEMVs).

Same function names, argument order, shapes and error behaviour as
`cuda_decode_gemv_ops/matvec.py:274-321` (`nosplit_matvec_half`) and
`cuda_decode_gemv_ops/fused.py:71-105, 261-337` (`fused_rmsnorm_qkv_half`,
`fused_post_attn_mlp_softsync_half`); the kernels behind them are the B200
persistent phase kernels of `libaicas_decode.so`.
"""
from __future__ import annotations

import torch

import _ops

__all__ = ["nosplit_matvec_half", "fused_rmsnorm_qkv_half", "fused_post_attn_mlp_softsync_half",
           "lm_head_argmax_half"]


def _decode_ok(*ts) -> bool:
    return all(t.device.type == "cuda" and t.dtype == torch.float16 for t in ts)


def nosplit_matvec_half(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                        workspace: dict | None = None) -> torch.Tensor:
    """y = x @ weight.T (+ bias) for one decode token (x [..., 1, k])."""
    if not _decode_ok(x, weight) or x.ndim < 2 or x.shape[-2] != 1:
        raise RuntimeError("nosplit_matvec_half expects fp16 CUDA single-token decode tensors")
    n, _k = weight.shape
    out = None
    if (workspace is not None and workspace.get("type") == "nosplit"
            and tuple(workspace["out"].shape) == (n,) and workspace["out"].device == x.device
            and workspace["out"].dtype == x.dtype):
        out = workspace["out"]
    out = _ops.gemv(x.reshape(-1).contiguous(), weight, bias, out=out)
    return out.view(*x.shape[:-1], n)


def fused_rmsnorm_qkv_half(x: torch.Tensor, norm_weight: torch.Tensor, weight: torch.Tensor,
                           bias: torch.Tensor | None, eps: float) -> torch.Tensor:
    """qkv = W_qkv @ RMSNorm(x) for one decode token."""
    if not _decode_ok(x, norm_weight, weight) or x.ndim < 2 or x.shape[-2] != 1:
        raise RuntimeError("fused_rmsnorm_qkv_half expects fp16 CUDA single-token decode tensors")
    n, _k = weight.shape
    out = _ops.gemv(x.reshape(-1).contiguous(), weight, bias, norm_w=norm_weight.reshape(-1).contiguous(),
                    eps=eps)
    return out.view(*x.shape[:-1], n)


def fused_post_attn_mlp_softsync_half(residual: torch.Tensor, attn_output: torch.Tensor,
                                      norm_weight: torch.Tensor, gate_up_weight: torch.Tensor,
                                      down_proj_weight: torch.Tensor, bias: torch.Tensor | None, eps: float,
                                      workspace: dict | None = None, threads_per_block: int = 1024,
                                      launch_blocks: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(act, out): h = residual + attn_output, act = SiLU(gate(RMSNorm h)) *
    up(RMSNorm h), out = h + down(act).  `threads_per_block` and
    `launch_blocks` are accepted for signature compatibility; the B200
    kernel always runs one 288-thread CTA per SM."""
    del threads_per_block, launch_blocks
    if (not _decode_ok(residual, attn_output, norm_weight, gate_up_weight, down_proj_weight)
            or residual.ndim < 2 or residual.shape[-2] != 1 or residual.shape != attn_output.shape):
        raise RuntimeError("fused_post_attn_mlp_softsync_half expects fp16 CUDA single-token decode tensors")
    n, inter = down_proj_weight.shape
    act, out = None, None
    if workspace is not None and workspace.get("type") == "fused_post_attn_mlp_softsync":
        act, out = workspace.get("hidden_out"), workspace.get("out")
    act, out = _ops.post_attn_mlp(residual.reshape(-1).contiguous(), attn_output.reshape(-1).contiguous(),
                                  norm_weight.reshape(-1).contiguous(), gate_up_weight, down_proj_weight,
                                  bias, eps, act_out=act, out=out)
    return act.view(*residual.shape[:-1], inter), out.view(*residual.shape[:-1], n)


def lm_head_argmax_half(x: torch.Tensor, weight: torch.Tensor, norm_weight: torch.Tensor | None = None,
                        eps: float = 1e-6, return_logits: bool = True):
    """Tied lm_head GEMV fused with the greedy argmax (the reference runs
    `nosplit_matvec_half` then `torch.argmax`, evaluation_wrapper.py:1233-1238
    and :952).  Returns (logits [..., vocab] or None, token [..., 1] int64)."""
    if not _decode_ok(x, weight) or x.shape[-2] != 1:
        raise RuntimeError("lm_head_argmax_half expects fp16 CUDA single-token decode tensors")
    logits, tok = _ops.lm_head_argmax(x.reshape(-1).contiguous(), weight,
                                      norm_w=None if norm_weight is None else norm_weight.reshape(-1),
                                      eps=eps, want_logits=return_logits)
    lead = x.shape[:-1]
    return (None if logits is None else logits.view(*lead, -1)), tok.view(*lead[:-1], 1)
