"""Checked one-call transport functions (reference: src/moe_dispatch/ops.py).

Each call validates its tensors before launching; the block and the
benchmarks skip that cost by calling a workspace's methods directly.
"""

from dataclasses import dataclass
import torch
from .workspace import CudaWorkspace, MAX_EXPERTS, MAX_TOPK


@dataclass(frozen=True)
class PackedTokens:
    """The dispatch results, as tensors that alias the workspace's buffers: the
    next dispatch into the same workspace overwrites them, so clone what must
    outlive it."""

    packed: torch.Tensor
    inverse: torch.Tensor
    counts: torch.Tensor
    offsets: torch.Tensor
    workspace: CudaWorkspace


def validate_inputs(x, expert_ids, experts, check_range=True):
    """ops.py:19-39, with the limits lifted to 1..512 experts and top-k 1..32.
    `check_range=False` skips the host-synchronising id range check."""
    if x.ndim != 2 or expert_ids.ndim != 2:
        raise ValueError("expected x[T,H] and expert_ids[T,K]")
    if x.shape[0] != expert_ids.shape[0] or x.shape[1] < 1:
        raise ValueError("token dimensions must match and H must be positive")
    if x.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise TypeError("x must be FP16, FP32, or BF16")
    if expert_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("expert_ids must be int32 or int64")
    if x.device != expert_ids.device:
        raise ValueError("x and expert_ids must be on the same device")
    if not x.is_contiguous() or not expert_ids.is_contiguous():
        raise ValueError("inputs must be contiguous")
    if not isinstance(experts, int) or not 1 <= experts <= MAX_EXPERTS:
        raise ValueError(f"experts must be an integer in 1..{MAX_EXPERTS}")
    if not 1 <= expert_ids.shape[1] <= MAX_TOPK:
        raise ValueError(f"topk must be 1..{MAX_TOPK}")
    if x.requires_grad:
        raise ValueError("CUDA operators are forward-only; detach inputs or use inference_mode")
    if check_range and expert_ids.numel() and (
            expert_ids.min().item() < 0 or expert_ids.max().item() >= experts):
        raise ValueError("expert_ids contains an out-of-range expert")


@torch.inference_mode()
def dispatch(x, expert_ids, experts, *, workspace=None, vectorized=True, alignment=1,
             check_range="host"):
    """Pack routed tokens by expert.

    check_range="host" (the reference's behaviour, ops.py:38) raises ValueError
    on an out-of-range id and synchronises.  "device" does not synchronise:
    such ids are skipped (slot and inverse -1) and counted on the device, in
    `workspace.invalid_ids_device` (read it with `workspace.invalid_ids()` or
    `raise_on_invalid_ids`), so the call can be captured in a CUDA graph.
    "none" skips the count's check entirely (the kernel still skips such ids).
    """
    if check_range not in ("host", "device", "none"):
        raise ValueError("check_range must be host, device or none")
    validate_inputs(x, expert_ids, experts, check_range=check_range == "host")
    if not x.is_cuda:
        raise RuntimeError("dispatch requires CUDA; the PyTorch reference runs on the CPU")
    expected_shape = (x.shape[0], x.shape[1], experts, expert_ids.shape[1])
    if workspace is None:
        workspace = CudaWorkspace(
            *expected_shape, x.dtype, vectorized=vectorized, device=x.device, alignment=alignment
        )
    if workspace.shape != expected_shape or workspace.dtype != x.dtype:
        raise ValueError("workspace shape/dtype does not match inputs")
    if workspace.packed.device != x.device:
        raise ValueError("workspace device does not match inputs")
    workspace.dispatch(x, expert_ids.to(torch.int32))
    return PackedTokens(
        workspace.packed, workspace.inverse, workspace.counts, workspace.offsets, workspace
    )


@torch.inference_mode()
def combine(expert_output, batch, weights):
    """out[t] = sum over k of weights[t,k] * expert_output[inverse[t,k]], summed in
    fp32 and cast once; the result is the workspace's output buffer, which the
    next combine overwrites."""
    if weights.shape != batch.inverse.shape:
        raise ValueError("weights must have shape [T,K]")
    if expert_output.shape != batch.packed.shape or expert_output.dtype != batch.packed.dtype:
        raise ValueError("expert output shape/dtype must match packed tokens")
    if weights.device != batch.packed.device or expert_output.device != batch.packed.device:
        raise ValueError("all tensors must be on the workspace device")
    if not weights.is_contiguous() or not expert_output.is_contiguous():
        raise ValueError("expert output and weights must be contiguous")
    if not weights.is_floating_point():
        raise TypeError("weights must be floating point")
    batch.workspace.combine(expert_output, weights.to(torch.float32))
    return batch.workspace.output


def raise_on_invalid_ids(batch):
    """After dispatch(check_range="device"): raise ValueError if the last
    dispatch saw out-of-range expert ids (synchronises)."""
    bad = batch.workspace.invalid_ids()
    if bad:
        raise ValueError(f"expert_ids contained {bad} out-of-range expert id(s)")
