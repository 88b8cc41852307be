"""CPU oracle for the training loss (test infrastructure, never the product).

Restates rwkv_mlx/train.py in float64 torch (autograd gives the exact gradients):
  * ``l2_wrap_loss``        : train.py:317-334  mean cross-entropy + 1e-4/(B*T) * 0.5 *
                              sum over positions of (max logit)^2
  * ``l2_wrap_loss_masked`` : train.py:337-362  the cross-entropy averaged over
                              mask = 1 positions (denominator sum(mask) + 1e-9), the
                              same L2 term over all positions
Pinned against the reference's own functions by tests/test_golden_oracle.py
(golden vectors from tests/golden/make_golden.py).
"""

from __future__ import annotations

import torch


def _ce(logits2d, targets1d):
    lse = torch.logsumexp(logits2d, dim=-1)
    return lse - logits2d.gather(-1, targets1d.long()[:, None])[:, 0]


def l2_wrap_loss(logits, targets):
    """logits (B, T, V), targets (B, T) -> scalar."""
    B, T, V = logits.shape
    ce = _ce(logits.reshape(-1, V), targets.reshape(-1)).mean()
    mx = logits.max(dim=-1).values
    return ce + 1e-4 / (B * T) * 0.5 * (mx ** 2).sum()


def l2_wrap_loss_masked(logits, targets, mask):
    B, T, V = logits.shape
    per = _ce(logits.reshape(-1, V), targets.reshape(-1))
    m = mask.reshape(-1).to(per.dtype)
    ce = (per * m).sum() / (m.sum() + 1e-9)
    mx = logits.max(dim=-1).values
    return ce + 1e-4 / (B * T) * 0.5 * (mx ** 2).sum()
