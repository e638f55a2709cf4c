"""A stack of MoE feed-forward layers with their pre-norms: the MoE half of the
reference's decoder layer (src/model/qwen35/decoder.rs:180-217) repeated,
x = RMSNorm(h) (src/ops/norm.rs:81-106), then h = h + MoE(x) with the
residual fused into the layer's combine. Device tensors, one stream, every
step through the C ABI (moe_b200_rms_norm, moe_b200_forward_device).
"""
from __future__ import annotations

import numpy as np

from ._lib import check

__all__ = ["MoeStack"]


class MoeStack:
    """layers: (Moe, Router) per layer (layers may share a bank);
    norm_weights: one [hidden] f32 RMSNorm weight per layer."""

    def __init__(self, layers, norm_weights, eps: float = 1e-6, zero_centered: bool = False,
                 device: int = 0):
        import torch
        if not layers or len(layers) != len(norm_weights):
            raise ValueError("one RMSNorm weight per layer")
        self.H = layers[0][0].hidden
        if any(moe.hidden != self.H for moe, _ in layers):
            raise ValueError("stack layers differ in hidden size")
        if not (np.isfinite(eps) and eps > 0):
            raise ValueError("invalid RMSNorm epsilon")
        self.layers = list(layers)
        self.lib = layers[0][0].owner.lib
        self.eps = float(eps)
        self.zero_centered = int(bool(zero_centered))
        self.device = torch.device("cuda", device)
        self.norms = []
        for w in norm_weights:
            w = np.ascontiguousarray(w, dtype=np.float32)
            if w.shape != (self.H,):
                raise ValueError("RMSNorm weight shape mismatch")
            self.norms.append(torch.from_numpy(w).to(self.device))

    @property
    def max_rows(self) -> int:
        return min(moe.max_rows() for moe, _ in self.layers)

    def rms_norm(self, d_x: int, d_weight: int, rows: int, d_out: int, stream: int) -> None:
        check(self.lib.moe_b200_rms_norm(d_x, d_weight, rows, self.H, self.eps, self.zero_centered,
                                         d_out, stream), "RMSNorm")

    def forward_tensor(self, h, out=None, stream: int | None = None):
        """h: [rows, hidden] f32 CUDA tensor (left unchanged). Returns the
        stack's output (`out` when given)."""
        import torch
        rows = h.shape[0]
        if h.dtype != torch.float32 or h.shape != (rows, self.H) or not h.is_contiguous():
            raise ValueError("stack input shape mismatch")
        if rows > self.max_rows:
            raise ValueError("rows above the layers' max_rows")
        s = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        x = torch.empty_like(h)
        bufs = (torch.empty_like(h), torch.empty_like(h))
        cur = h
        for i, ((moe, router), w) in enumerate(zip(self.layers, self.norms)):
            self.rms_norm(cur.data_ptr(), w.data_ptr(), rows, x.data_ptr(), s)
            nxt = bufs[i % 2]
            moe.forward_device(router, rows, x.data_ptr(), cur.data_ptr(), nxt.data_ptr(), s)
            cur = nxt
        if out is None:
            return cur
        out.copy_(cur)
        return out

    def forward(self, h: np.ndarray) -> np.ndarray:
        """Host convenience: [rows, hidden] f32 in, the stack's output out."""
        import torch
        t = torch.from_numpy(np.ascontiguousarray(h, dtype=np.float32)).to(self.device)
        out = self.forward_tensor(t)
        torch.cuda.synchronize(self.device)
        for moe, _ in self.layers:
            moe.status()
        return out.cpu().numpy()
