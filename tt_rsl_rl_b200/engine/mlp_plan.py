"""Device execution plan of one MLP (Linear + ELU stack) on the tcgen05 GEMM.

For a model ``MLPModel.mlp`` with layers ``W_1 .. W_L`` it owns bf16 weight shadows, activation buffers for a rollout
batch and a training minibatch, and the partial-gradient buffers, and issues:

* forward      ``H_l = elu(H_{l-1} W_l^T + b_l)`` (bf16 activations kept for backward), last layer fp32;
* backward     data gradients ``dZ_{l-1} = (dZ_l W_l) * elu'(H_{l-1})`` with per-CTA column sums (bias gradients)
               and weight gradients ``dW_l = dZ_l^T H_{l-1}`` as split-K fp32 partials.

Row pitches of all bf16 buffers are padded to multiples of 8 elements (16 bytes, the TMA stride rule).
The math follows ``rsl_rl/modules/mlp.py:91-95`` (forward) and its autograd backward.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..ops import ext
from ..ops import gemm as G


def pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def wgrad_splits(out_f: int, in_f: int, rows: int, sm_count: int) -> int:
    """Split-K factor so the weight-gradient GEMM fills the GPU once (about one CTA per SM)."""
    bn = 64 if in_f <= 64 else 128 if in_f <= 128 else 256
    tiles = ((out_f + 127) // 128) * ((in_f + bn - 1) // bn)
    kb = (rows + 63) // 64
    return max(1, min(kb, sm_count // max(1, tiles)))


class MLPPlan:
    def __init__(self, mlp: nn.Module, in_dim: int, rows_roll: int, rows_train: int, device: torch.device,
                 sm_count: int, train: bool = True, grads: bool = True) -> None:
        self.linears: list[nn.Linear] = [m for m in mlp if isinstance(m, nn.Linear)]
        self.L = len(self.linears)
        self.widths = [in_dim] + [lin.out_features for lin in self.linears]
        if self.linears[0].in_features != in_dim:
            raise ValueError("MLP input width does not match the observation dimension")
        self.head_cols = self.widths[-1]
        self.device = device
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        # bf16 weight shadows [out, pad8(in)] (padding columns stay zero)
        self.w_bf16 = [torch.zeros(lin.out_features, pad8(lin.in_features), **bf) for lin in self.linears]
        self.rows_roll = rows_roll
        self.rows_train = rows_train
        # rollout activations
        self.x_roll = torch.zeros(rows_roll, pad8(in_dim), **bf)
        self.h_roll = [torch.zeros(rows_roll, pad8(w), **bf) for w in self.widths[1:-1]]
        # head outputs with the row pitch rounded up to 32 columns: the head GEMM then stores whole 32-column chunks
        # (the padding columns hold zeros); consumers read them at this pitch (``out.shape[1]``)
        self.out_pitch = (self.head_cols + 31) // 32 * 32
        self.out_roll = torch.zeros(rows_roll, self.out_pitch, **f32)
        self.train = train
        if not train:
            return
        B = rows_train
        self.x_train = torch.zeros(B, pad8(in_dim), **bf)
        self.h_train = [torch.zeros(B, pad8(w), **bf) for w in self.widths[1:-1]]
        self.out_train = torch.zeros(B, self.out_pitch, **f32)
        self.grads = grads
        if not grads:  # inference-only training-size buffers (a frozen network evaluated on minibatches)
            return
        # gradient of the head output (written by the loss kernel) and of hidden pre-activations
        self.d_head = torch.zeros(B, pad8(self.head_cols), **bf)
        self.dz = [torch.zeros(B, pad8(w), **bf) for w in self.widths[1:-1]]
        # bias-gradient partials of hidden layers: per-CTA column sums from the data-gradient GEMM of the next layer
        self.colsum_rows = int(ext().gemm_colsum_rows(sm_count))
        self.bias_partial = [torch.zeros(self.colsum_rows, w, **f32) for w in self.widths[1:-1]]
        self.splits = []
        self.wgrad_partial = []
        for lin in self.linears:
            s = wgrad_splits(lin.out_features, lin.in_features, B, sm_count)
            self.splits.append(s)
            self.wgrad_partial.append(torch.zeros(s, lin.out_features, lin.in_features, **f32))

    # ---- parameters -----------------------------------------------------------------------------------------------
    def refresh_shadows(self) -> None:
        """Re-derive the bf16 shadows from the fp32 master weights (after init or a checkpoint load)."""
        for lin, wb in zip(self.linears, self.w_bf16):
            ext().to_bf16_padded(lin.weight.data, wb, wb.shape[1])

    # ---- forward ----------------------------------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, hs: list[torch.Tensor], rows: int, out: torch.Tensor, out_ld: int,
                status: torch.Tensor | None = None) -> None:
        """x [rows, pad8(in)] bf16 -> hidden bf16 buffers hs -> out fp32 [rows, out_ld] (head, with bias)."""
        src = x
        for l, lin in enumerate(self.linears):
            K = self.widths[l]
            N = self.widths[l + 1]
            w = self.w_bf16[l]
            if l < self.L - 1:
                dst = hs[l]
                G.gemm(src, src.shape[1], False, w, w.shape[1], False, rows, N, K, G.EPI_BIAS_ELU_BF16, dst,
                       dst.shape[1], bias=lin.bias.data, status=status)
                src = dst
            else:
                # the plan's own head buffers may take whole 32-column chunks (their padding is this plan's)
                own = out is self.out_roll or (self.train and out is self.out_train)
                G.gemm(src, src.shape[1], False, w, w.shape[1], False, rows, N, K, G.EPI_F32, out, out_ld,
                       bias=lin.bias.data, status=status, out_cols=out_ld if own and out_ld >= N else 0)

    # ---- backward ---------------------------------------------------------------------------------------------------
    def backward(self, rows: int, status: torch.Tensor | None = None, x: torch.Tensor | None = None,
                 dx_out: torch.Tensor | None = None) -> None:
        """Weight gradients (split partials) of every layer and data gradients down to layer 1.

        Requires ``d_head`` (gradient of the head output, padding columns zero) and the cached activations of the
        training forward pass; ``x`` is that pass's input when it was not ``x_train``. With ``dx_out`` (fp32
        [rows, in_dim]) the gradient of the input, ``dZ_1 W_1``, is written as well (no activation below the input).
        """
        inputs = [self.x_train if x is None else x] + self.h_train  # input of layer l is inputs[l]
        dz_l = self.d_head
        for l in range(self.L - 1, -1, -1):
            lin = self.linears[l]
            out_f, in_f = lin.out_features, lin.in_features
            h_in = inputs[l]
            part = self.wgrad_partial[l]
            splits = min(self.splits[l], (rows + 63) // 64)
            if splits < self.splits[l]:  # a shorter minibatch: unused split partials must not keep stale sums
                part[splits:].zero_()
            # dW_l = dZ_l^T H_{l-1}: both operands read MN-major from row-major [rows, features] buffers
            G.gemm(dz_l, dz_l.shape[1], True, h_in, h_in.shape[1], True, out_f, in_f, rows, G.EPI_PARTIAL_F32, part,
                   in_f, splits=splits, split_stride=out_f * in_f, status=status)
            if l == 0:
                if dx_out is not None:
                    w = self.w_bf16[0]
                    G.gemm(dz_l, dz_l.shape[1], False, w, w.shape[1], True, rows, in_f, out_f, G.EPI_F32, dx_out,
                           dx_out.stride(0), status=status)
                break
            # dZ_{l-1} = (dZ_l W_l) * elu'(H_{l-1}); W_l [out, pad8(in)] read MN-major
            w = self.w_bf16[l]
            dz_prev = self.dz[l - 1]
            colsum = self.bias_partial[l - 1]  # every row written by the launch (unused CTAs' rows cleared)
            G.gemm(dz_l, dz_l.shape[1], False, w, w.shape[1], True, rows, in_f, out_f, G.EPI_DGRAD_ELU, dz_prev,
                   dz_prev.shape[1], aux=h_in, ld_aux=h_in.shape[1], colsum=colsum, status=status)
            dz_l = dz_prev

    # ---- gradient reduction segments ----------------------------------------------------------------------------------
    def reduce_segments(self, head_bias_partial: torch.Tensor, head_parts: int) -> dict[int, tuple]:
        """Map ``id(param)`` -> (partial buffer, parts, numel) for the weights and biases of this MLP."""
        segs = {}
        for l, lin in enumerate(self.linears):
            segs[id(lin.weight)] = (self.wgrad_partial[l], self.splits[l], lin.weight.numel())
            if l < self.L - 1:
                segs[id(lin.bias)] = (self.bias_partial[l], self.colsum_rows, lin.bias.numel())
            else:
                segs[id(lin.bias)] = (head_bias_partial, head_parts, lin.bias.numel())
        return segs
