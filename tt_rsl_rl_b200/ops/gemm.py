"""Thin Python wrappers around the tcgen05 GEMM (``csrc/gemm_tcgen05.cu``).

All matrices are row-major with a leading dimension (row pitch) in elements; bf16 pitches must be multiples of 8.
The three roles (forward with bias + ELU, data gradient with ELU', weight gradient) are the ``nn.Linear`` + ELU
stack of ``rsl_rl/modules/mlp.py:16-95`` and its autograd backward; the reference plugin writes the same VJP by hand
(``rsl_rl_tt/modules.py:160-262``).
"""

from __future__ import annotations

import torch

from . import ext

EPI_F32 = 0
EPI_BIAS_ELU_BF16 = 1
EPI_BIAS_BF16 = 2
EPI_DGRAD_ELU = 3
EPI_PARTIAL_F32 = 4


def pad8(n: int) -> int:
    """Round a bf16 row length up to the 16-byte TMA pitch rule."""
    return (n + 7) // 8 * 8


def m_tiles(m: int) -> int:
    """Number of 128-row tiles."""
    return (m + 127) // 128


def colsum_rows(device: torch.device | int | None = None) -> int:
    """Rows of a column-sum partial buffer of the data-gradient epilogue: one per CTA of the largest launch."""
    dev = torch.device("cuda") if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    return int(ext().gemm_colsum_rows(torch.cuda.get_device_properties(idx).multi_processor_count))


def gemm(
    a: torch.Tensor,
    lda: int,
    a_mn: bool,
    b: torch.Tensor,
    ldb: int,
    b_mn: bool,
    M: int,
    N: int,
    K: int,
    epilogue: int,
    out: torch.Tensor,
    ldo: int,
    *,
    splits: int = 1,
    split_stride: int = 0,
    bias: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    ld_aux: int = 0,
    colsum: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
    out_cols: int = 0,
) -> None:
    """out[M, N] = sum_k A(m, k) B(n, k) with the selected epilogue (see ``gemm_tcgen05.cuh``). ``out_cols`` (fp32
    outputs): columns of each row that may be written, N .. ldo (padding columns receive zeros)."""
    ext().gemm(a, lda, a_mn, b, ldb, b_mn, M, N, K, epilogue, out, ldo, splits, split_stride, bias, aux, ld_aux,
               colsum, status, out_cols)


def linear_forward(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, out: torch.Tensor, *, elu: bool,
                   ldx: int | None = None, ldw: int | None = None, ldo: int | None = None, k: int | None = None,
                   status: torch.Tensor | None = None) -> None:
    """out = act(x @ w.T + bias) with x [M, K] bf16, w [N, K] bf16; bf16 out for ELU layers, fp32 otherwise."""
    M = x.shape[0]
    N = w.shape[0]
    K = k if k is not None else x.shape[1]
    ldx = ldx if ldx is not None else x.stride(0)
    ldw = ldw if ldw is not None else w.stride(0)
    ldo = ldo if ldo is not None else out.stride(0)
    if elu:
        epi = EPI_BIAS_ELU_BF16
    else:
        epi = EPI_F32 if out.dtype == torch.float32 else EPI_BIAS_BF16
    gemm(x, ldx, False, w, ldw, False, M, N, K, epi, out, ldo, bias=bias, status=status)
