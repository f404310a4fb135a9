"""Reusable GPU buffers for dispatch/combine (reference: src/moe_dispatch/workspace.py).

One workspace per independent concurrent invocation: calls that share a
workspace (its buffers or its dispatch scratch) must not overlap in time.
"""

import torch
from ._extension import get_extension

MAX_EXPERTS = 512
MAX_TOPK = 32


def capacity_rows(tokens, experts, topk, alignment):
    """workspace.py:30-34: packed rows for `tokens*topk` assignments at `alignment`."""
    n = tokens * topk
    if alignment == 1:
        return n
    return (n + experts * (alignment - 1) + 1 + alignment - 1) // alignment * alignment


class CudaWorkspace:
    """Owns counts[E], offsets[E+1], slots[T*K], packed[R,H], inverse[T,K], output[T,H].

    Same constructor and methods as the reference's CudaWorkspace
    (workspace.py:7-87); the expert/top-k limits are 1..512 experts and
    top-k 1..32 instead of 1..64 and 1..2.
    """

    def __init__(
        self,
        tokens,
        hidden,
        experts,
        topk,
        dtype,
        vectorized=True,
        device="cuda",
        extension=None,
        alignment=1,
    ):
        if (
            tokens < 0
            or hidden < 1
            or experts < 1
            or experts > MAX_EXPERTS
            or not 1 <= topk <= MAX_TOPK
        ):
            raise ValueError(
                f"supports T>=0, H>=1, 1..{MAX_EXPERTS} experts, and topk=1..{MAX_TOPK}"
            )
        if tokens * topk > 2**31 - 1 or hidden > 2**31 - 1:
            raise ValueError("shape exceeds int32 indexing capacity")
        if dtype not in (torch.float16, torch.float32, torch.bfloat16):
            raise ValueError("CUDA workspace supports FP16, FP32, and BF16")
        if not 1 <= alignment <= 128:
            raise ValueError("alignment must be 1..128")
        self.alignment = alignment
        self.capacity_rows = capacity_rows(tokens, experts, topk, alignment)
        if self.capacity_rows > 2**31 - 1:
            raise ValueError("padded capacity exceeds int32 indexing capacity")
        device = torch.device(device)
        if device.type != "cuda" or not torch.cuda.is_available():
            raise RuntimeError("CudaWorkspace requires an NVIDIA CUDA GPU")
        self.shape = (tokens, hidden, experts, topk)
        self.dtype = dtype
        self.device = device
        self.vectorized = vectorized
        with torch.cuda.device(device):
            self.extension = extension if extension is not None else get_extension()
            self.counts = torch.empty(experts, device=device, dtype=torch.int32)
            self.offsets = torch.empty(experts + 1, device=device, dtype=torch.int32)
            self.slots = torch.empty(tokens * topk, device=device, dtype=torch.int32)
            self.packed = torch.empty((self.capacity_rows, hidden), device=device, dtype=dtype)
            self.inverse = torch.empty((tokens, topk), device=device, dtype=torch.int32)
            self.output = torch.empty((tokens, hidden), device=device, dtype=dtype)
            self.scratch = self.extension.make_scratch(tokens, topk, experts, device)

    def dispatch(self, x, ids32, ids64=None):
        """Pack x by expert without argument checks (the block's path): ids32 must be
        contiguous int32 in [0, experts) and x contiguous, of the workspace's shape."""
        if self.alignment == 1:
            self.extension.dispatch_out(
                x, ids32, self.counts, self.offsets, self.slots, self.packed, self.inverse,
                self.vectorized, scratch=self.scratch,
            )
        else:
            self.extension.dispatch_aligned_out(
                x, ids32, self.counts, self.offsets, self.slots, self.packed, self.inverse,
                self.vectorized, self.alignment, scratch=self.scratch,
            )

    @property
    def invalid_ids_device(self):
        """Device int32 [1]: out-of-range expert ids seen by the last dispatch
        (written by the index kernel; reading it on the device needs no sync)."""
        return self.scratch[2:3]

    def invalid_ids(self):
        """Out-of-range expert ids of the last dispatch (synchronises)."""
        return int(self.scratch[2].item())

    def combine(self, expert_output, weights, out=None):
        """Weighted sum of each token's K expert rows into `out` (default: self.output)."""
        out = self.output if out is None else out
        self.extension.combine_out(expert_output, self.inverse, weights, out)
        return out

    @property
    def workspace_bytes(self):
        return sum(
            t.numel() * t.element_size()
            for t in [self.counts, self.offsets, self.slots, self.packed, self.inverse,
                      self.output, self.scratch]
        )
