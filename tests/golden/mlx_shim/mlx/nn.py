"""mlx.nn stand-in (numpy).  Fixture generation only."""

import numpy as np


class Module:
    def __call__(self, *args, **kwargs):  # subclasses define __call__
        raise NotImplementedError


class Linear(Module):
    def __init__(self, input_dims, output_dims, bias=True):
        self.weight = np.zeros((output_dims, input_dims), np.float32)
        if bias:
            self.bias = np.zeros((output_dims,), np.float32)

    def __call__(self, x):
        y = x @ self.weight.T
        return y + self.bias if hasattr(self, "bias") else y


class Embedding(Module):
    def __init__(self, num_embeddings, dims):
        self.weight = np.zeros((num_embeddings, dims), np.float32)

    def __call__(self, idx):
        return self.weight[np.asarray(idx)]


class LayerNorm(Module):
    def __init__(self, dims, eps=1e-5, affine=True, bias=True):
        self.eps = eps
        self.weight = np.ones((dims,), np.float32)
        self.bias = np.zeros((dims,), np.float32)

    def __call__(self, x):
        m = x.mean(-1, keepdims=True)
        v = ((x - m) ** 2).mean(-1, keepdims=True)
        return ((x - m) / np.sqrt(v + self.eps)) * self.weight + self.bias


class GroupNorm(Module):
    """MLX GroupNorm.  With the default pytorch_compatible=False MLX reshapes the
    input to (batch, -1, num_groups) and normalises over axis 1, so group g holds
    the channels c with c % num_groups == g."""

    def __init__(self, num_groups, dims, eps=1e-5, affine=True, pytorch_compatible=False):
        self.num_groups, self.dims, self.eps, self.pc = num_groups, dims, eps, pytorch_compatible
        self.weight = np.ones((dims,), np.float32)
        self.bias = np.zeros((dims,), np.float32)

    def __call__(self, x):
        batch, *rest, dims = x.shape
        G = self.num_groups
        if self.pc:
            gs = dims // G
            xg = x.reshape(batch, -1, G, gs).transpose(0, 2, 1, 3).reshape(batch, G, -1)
            m = xg.mean(-1, keepdims=True)
            v = xg.var(-1, keepdims=True)
            y = (xg - m) / np.sqrt(v + self.eps)
            y = y.reshape(batch, G, -1, gs).transpose(0, 2, 1, 3).reshape(batch, *rest, dims)
        else:
            xg = x.reshape(batch, -1, G)
            m = xg.mean(axis=1, keepdims=True)
            v = xg.var(axis=1, keepdims=True)
            y = ((xg - m) / np.sqrt(v + self.eps)).reshape(batch, *rest, dims)
        return self.weight * y + self.bias


def softplus(x):
    return np.logaddexp(x, 0).astype(x.dtype)


def relu(x):
    return np.maximum(x, 0)


class losses:
    """mlx.nn.losses subset."""

    @staticmethod
    def cross_entropy(logits, targets, reduction="none"):
        """-log softmax(logits)[target] per row (MLX's documented definition, class
        axis last), then the reduction ("none" | "mean" | "sum")."""
        lg = np.asarray(logits, np.float64)
        m = lg.max(axis=-1, keepdims=True)
        lse = (m + np.log(np.exp(lg - m).sum(axis=-1, keepdims=True)))[..., 0]
        tgt = np.take_along_axis(lg, np.asarray(targets).astype(np.int64)[..., None], axis=-1)[..., 0]
        loss = (lse - tgt).astype(np.asarray(logits).dtype)
        if reduction == "mean":
            return loss.mean()
        if reduction == "sum":
            return loss.sum()
        return loss
