"""`QuantizedLinear`: a 4-bit MLX-affine projection as a torch module (the counterpart of mlx.nn's
QuantizedLinear that the reference's qmv modules swap, ironmule/qmv_k3840.py:313-342). Its forward runs the
B200 qGEMM for every input shape: rows are taken 32 at a time (the warp-MMA kernel's limit); there is no
library or CPU path.
"""
from __future__ import annotations

import torch

from . import kernels

GROUP_SIZE = 64
BITS = 4
MAX_ROWS_PER_CALL = 32


class QuantizedLinear(torch.nn.Module):
    """weight int32 [N, K/8] (uint32 bit patterns), scales/biases bf16 [N, K/64], group 64, 4 bits."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 group_size: int = GROUP_SIZE, bits: int = BITS):
        super().__init__()
        if group_size != GROUP_SIZE or bits != BITS:
            raise ValueError("only 4-bit, group-64 affine weights are supported")
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group_size, self.bits = group_size, bits

    @classmethod
    def from_linear(cls, weight: torch.Tensor) -> "QuantizedLinear":
        """Quantise a bf16 [N, K] weight on its (CUDA) device."""
        wq, s, b = kernels.quantize(weight.to(torch.bfloat16).contiguous())
        return cls(wq, s, b)

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[1]) * 32 // self.bits

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        rows = x2.shape[0]
        if rows <= MAX_ROWS_PER_CALL:
            y = kernels.qgemm(x2, self.weight, self.scales, self.biases)
        else:
            y = torch.empty((rows, self.out_features), dtype=torch.bfloat16, device=x.device)
            for r in range(0, rows, MAX_ROWS_PER_CALL):
                part = x2[r:r + MAX_ROWS_PER_CALL]
                kernels.qgemm(part, self.weight, self.scales, self.biases, out=y[r:r + part.shape[0]])
        return y.view(*lead, self.out_features)
