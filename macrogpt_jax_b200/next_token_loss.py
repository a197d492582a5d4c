"""Next-token prediction loss (ueaj/opt/next_token_loss.py) on this package's kernels.

Same names, arguments and results as the reference module:
  ntp_loss_mask(inputs, document_ids, pad_token_id, loss_mask)        next_token_loss.py:13-58
  ntp_args(inputs, document_ids, pad_token_id, loss_mask)             next_token_loss.py:61-97
  chunked_softmax_cross_entropy(inputs, activations, logit_projection, chunk_size, document_ids,
                                pad_token_id, loss_mask, return_loss_mask, **kwargs)  :99-174
  softmax_cross_entropy_with_integer_labels(logits, labels)   (optax's, which the reference calls)

chunked_softmax_cross_entropy returns the per-token loss [batch, seq] (masked positions 0), f32
where the reference returns the logits' dtype (bf16).  Two paths:
  * `logit_projection` is an OutputHead (or its get_logits / forward) whose norm and lm_head are
    this package's RMSNorm and FP8 Einsum: the fused node of head.py over all tokens at once.  The
    reference chunks the sequence to bound the memory of the logits; on a 180 GB device the bf16
    logits of a whole batch fit (4.2 GB for 16384 tokens x 128256 classes), and the per-tensor fp8
    scales are then those of the whole call.  `chunk_size` is accepted and not needed.
  * any other projection: the reference's chunking (chunks of `chunk_size` positions along the
    sequence, a shorter last chunk), each chunk's logits computed by the projection under
    activation checkpointing (the reference's use_checkpointing=True) and its loss by
    ufp8_xent_forward / ufp8_xent_backward on the bf16 logits.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.utils.checkpoint

from . import _capi as C
from . import ops
from .head import OutputHead


def ntp_loss_mask(inputs: torch.Tensor, document_ids: Optional[torch.Tensor] = None,
                  pad_token_id: Optional[int] = None, loss_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Binary mask [batch, seq]: 0 at the last position, where the next token is padding, and
    where the next token starts another document; times loss_mask."""
    mask = torch.ones(inputs.shape[:2], dtype=torch.int32, device=inputs.device)
    mask[:, -1] = 0
    if loss_mask is not None:
        mask = mask * loss_mask.to(torch.int32)
    if pad_token_id is not None:
        mask[:, :-1] *= (inputs[:, 1:] != pad_token_id).to(torch.int32)
    if document_ids is not None:
        mask[:, :-1] *= (document_ids[:, :-1] == document_ids[:, 1:]).to(torch.int32)
    return mask


def ntp_args(inputs: torch.Tensor, document_ids: Optional[torch.Tensor] = None, pad_token_id: Optional[int] = None,
             loss_mask: Optional[torch.Tensor] = None):
    """(targets, mask): targets[:, i] = inputs[:, i + 1]; the last position keeps its own token."""
    mask = ntp_loss_mask(inputs, document_ids, pad_token_id, loss_mask)
    targets = inputs.clone()
    targets[:, :-1] = inputs[:, 1:]
    return targets, mask


class _XentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits2d, labels, mask):
        lse, loss, _ = ops.xent_rows(logits2d, labels, mask)
        ctx.save_for_backward(logits2d, labels, mask, lse)
        return loss

    @staticmethod
    def backward(ctx, dloss):
        logits2d, labels, mask, lse = ctx.saved_tensors
        dl = ops.xent_grad(logits2d, labels, mask, lse, None, dloss.to(torch.float32).contiguous(), 0.0, C.BF16)
        return dl, None, None


def _token_loss(logits: torch.Tensor, labels: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    if logits.dtype != torch.bfloat16:
        raise TypeError(f"the cross-entropy kernels take bf16 logits (the lm_head's output dtype), got {logits.dtype}")
    lead = logits.shape[:-1]
    l2d = logits.reshape(-1, logits.shape[-1])
    if l2d.stride(-1) != 1:
        l2d = l2d.contiguous()
    lab = labels.reshape(-1).to(torch.int32).contiguous()
    mk = None if mask is None else mask.reshape(-1).to(torch.uint8).contiguous()
    return _XentFn.apply(l2d, lab, mk).reshape(lead)


def softmax_cross_entropy_with_integer_labels(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """logsumexp(logits) - logits[label] over the last axis (optax's function), f32 result."""
    return _token_loss(logits, labels, None)


def _fused_head(logit_projection) -> Optional[OutputHead]:
    head = getattr(logit_projection, "__self__", logit_projection)
    if not isinstance(head, OutputHead) or not head.fused():
        return None
    fn = getattr(logit_projection, "__func__", None)
    if logit_projection is head or fn in (OutputHead.get_logits, OutputHead.forward):
        return head
    return None


def chunked_softmax_cross_entropy(inputs: torch.Tensor, activations: torch.Tensor,
                                  logit_projection: Callable[..., torch.Tensor], chunk_size: int = 1024,
                                  document_ids: Optional[torch.Tensor] = None, pad_token_id: Optional[int] = None,
                                  loss_mask: Optional[torch.Tensor] = None, return_loss_mask: bool = False,
                                  **logit_proj_kwargs):
    """Per-token next-token loss [batch, seq] (see the module docstring for the two paths)."""
    targets, mask = ntp_args(inputs, loss_mask=loss_mask, document_ids=document_ids, pad_token_id=pad_token_id)
    head = _fused_head(logit_projection) if not logit_proj_kwargs else None
    if head is not None:
        out = head.token_loss(activations, targets, mask)
    else:
        seq = activations.shape[1]

        def chunk_loss(act, tgt, mk):
            return _token_loss(logit_projection(act, **logit_proj_kwargs), tgt, mk)

        pieces = []
        for s in range(0, seq, chunk_size):
            e = min(s + chunk_size, seq)
            args = (activations[:, s:e], targets[:, s:e], mask[:, s:e])
            if torch.is_grad_enabled():
                pieces.append(torch.utils.checkpoint.checkpoint(chunk_loss, *args, use_reentrant=False))
            else:
                pieces.append(chunk_loss(*args))
        out = torch.cat(pieces, dim=1)
    if return_loss_mask:
        return out, mask
    return out
