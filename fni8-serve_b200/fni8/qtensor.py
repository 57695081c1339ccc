"""QTensor: the quantized-weight container fni8-serve's layers consume.

Same constructor and attributes as the external type the reference imports
(`QTensor(data, scale, scheme=, group_size=, codebook=)`, used at
fni8serve/models/weights.py:25,37 and fni8serve/loader.py:95). For `per_row_i8`,
`data` is int8 [out_features, in_features] (K contiguous) and `scale` fp32
[out_features]: one symmetric scale per output channel, the layout the tcgen05 GEMM
reads directly as its B operand (no repack).
"""
from __future__ import annotations

import torch

SCHEMES = ("per_row_i8", "per_group_i4", "raw")


class QTensor:
    def __init__(self, data: torch.Tensor, scale: torch.Tensor | None, scheme: str = "per_row_i8",
                 group_size: int | None = None, codebook: str | None = None):
        if scheme not in SCHEMES:
            raise ValueError(f"unknown QTensor scheme {scheme!r}")
        self.data = data
        self.scale = scale
        self.scheme = scheme
        self.group_size = group_size
        self.codebook = codebook

    @property
    def shape(self) -> torch.Size:
        return self.data.shape

    @property
    def device(self) -> torch.device:
        return self.data.device

    def to(self, device) -> "QTensor":
        return QTensor(self.data.to(device), None if self.scale is None else self.scale.to(device), self.scheme,
                       self.group_size, self.codebook)

    def cuda(self, device=None) -> "QTensor":
        return self.to(torch.device("cuda") if device is None else device)

    def __repr__(self) -> str:
        return (f"QTensor(scheme={self.scheme}, shape={tuple(self.data.shape)}, dtype={self.data.dtype}, "
                f"device={self.data.device})")
