"""MoE feed-forward block on B200 kernels (reference: src/moe_dispatch/layer.py).

Same public surface as the reference -- ``MoEConfig``, ``MoEWeights``,
``make_weights``, ``MoEBlock`` with ``forward``, ``route``, ``workspace``,
``experts_forward``, ``set_routing_pattern`` -- with the expert/top-k limits
raised to the configurations this engine targets (up to 256 experts, top-k up
to 32).  Every stage runs a kernel from libmoe_b200.so:

  route            moe_route: fp32 logits + top-k + softmax
  dispatch         moe_dispatch: histogram/scan/pack, aligned spans
  experts_forward  cuda_fused: tcgen05 gate/up GEMM with SwiGLU epilogue,
                   then the tcgen05 down GEMM;
                   cuda: plain gate/up GEMM, swiglu kernel, down GEMM;
                   expert_dtype="fp8_e4m3" (an extension: the reference's
                   experts are bf16 only): per-row e4m3 activations and
                   per-channel e4m3 gate/up weights on tcgen05.kind::f8f6f4,
                   dequantised in the epilogue; the down GEMM stays bf16
  combine          moe_combine
"""

from dataclasses import dataclass
import math
import torch
from .workspace import CudaWorkspace
from ._extension import get_extension

MAX_EXPERTS = 256
MAX_TOPK = 32


@dataclass(frozen=True)
class MoEConfig:
    hidden: int = 512
    intermediate: int = 1024
    experts: int = 8
    topk: int = 2
    alignment: int = 8

    def __post_init__(self):
        if self.hidden < 8 or self.intermediate < 8:
            raise ValueError("hidden/intermediate must be at least 8")
        if self.hidden % 8 or self.intermediate % 8:
            raise ValueError("grouped GEMM dimensions must be multiples of 8")
        if (
            not 1 <= self.experts <= MAX_EXPERTS
            or not 1 <= self.topk <= MAX_TOPK
            or self.topk > self.experts
        ):
            raise ValueError("invalid expert/topk configuration")
        if not 8 <= self.alignment <= 128 or self.alignment % 8:
            raise ValueError("full-block grouped GEMM alignment must be a multiple of 8 up to 128")


@dataclass
class MoEWeights:
    router: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor


def make_weights(config, device, dtype, seed=42):
    """Seeded weights drawn in the reference's order (layer.py:38-59).

    router [E,H] fp32 ~ N(0,1)/sqrt(H); gate_up [E,2I,H] ~ N(0,1)/sqrt(H) (gate
    rows 0..I-1, up rows I..2I-1); down [E,H,I] ~ N(0,1)/sqrt(I); one generator
    on `device`, so the bytes match the reference's for the same device and seed.
    """
    generator = torch.Generator(device=device).manual_seed(seed)
    router = torch.randn(
        config.experts, config.hidden, device=device, generator=generator
    ) / math.sqrt(config.hidden)
    gate_up = (
        torch.randn(
            config.experts, 2 * config.intermediate, config.hidden, device=device,
            generator=generator,
        )
        / math.sqrt(config.hidden)
    ).to(dtype)
    down = (
        torch.randn(
            config.experts, config.hidden, config.intermediate, device=device, generator=generator
        )
        / math.sqrt(config.intermediate)
    ).to(dtype)
    return MoEWeights(router, gate_up, down)


@dataclass
class LayerWorkspace:
    transport: object
    projection: torch.Tensor
    activated: torch.Tensor
    expert_output: torch.Tensor
    packed_q: torch.Tensor = None      # e4m3 copy of the packed rows (expert_dtype="fp8_e4m3")
    packed_scale: torch.Tensor = None  # their per-row dequantisation scales


def check_out(out, x):
    """Reject an explicit output buffer that the combine cannot write as-is."""
    if out is None:
        return
    if (out.shape != x.shape or out.dtype != x.dtype or out.device != x.device
            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous tensor with x's shape, dtype and device")


class MoEBlock(torch.nn.Module):
    """A forward-only mixture-of-experts feed-forward layer on the B200 kernels.

    Each forward routes every token to its top-k experts, packs the rows by
    expert, runs the gate/up and down grouped GEMMs (SwiGLU between them) and
    sums each token's expert rows weighted by its routing weights.
    `cuda_fused` applies SwiGLU in the gate/up GEMM's epilogue; `cuda` writes
    the bf16 projection and runs the standalone SwiGLU kernel.  Both round at
    the same points, so they produce the same bits.  Without `out=` the result
    lives in a buffer the next forward of the same shape reuses.
    """

    def __init__(
        self,
        config=None,
        *,
        device="cuda",
        dtype=torch.bfloat16,
        implementation="cuda_fused",
        expert_backend="auto",
        seed=42,
        weights=None,
        expert_dtype="bf16",
    ):
        super().__init__()
        self.config = config or MoEConfig()
        if expert_dtype not in ("bf16", "fp8_e4m3"):
            raise ValueError("expert_dtype must be bf16 or fp8_e4m3")
        if expert_dtype == "fp8_e4m3" and self.config.hidden % 16:
            raise ValueError("fp8_e4m3 experts need hidden to be a multiple of 16")
        self.expert_dtype = expert_dtype
        if implementation == "torch":
            raise ValueError(
                "this engine has CUDA implementations only (cuda, cuda_fused); the PyTorch "
                "path is the reference's"
            )
        if implementation not in ("cuda", "cuda_fused"):
            raise ValueError("implementation must be cuda or cuda_fused")
        if expert_backend not in ("auto", "tcgen05"):
            raise ValueError("expert backend must be auto or tcgen05 (the only GEMM here)")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("CUDA implementations require CUDA")
        if dtype != torch.bfloat16:
            raise ValueError("full CUDA block uses BF16 grouped GEMMs")
        self.implementation = implementation
        self.expert_backend = "tcgen05"
        weights = weights or make_weights(self.config, device, dtype, seed)
        expected_gate = (self.config.experts, 2 * self.config.intermediate, self.config.hidden)
        expected_down = (self.config.experts, self.config.hidden, self.config.intermediate)
        if tuple(weights.gate_up.shape) != expected_gate or tuple(weights.down.shape) != expected_down:
            raise ValueError("expert weights do not match the block configuration")
        if tuple(weights.router.shape) != (self.config.experts, self.config.hidden):
            raise ValueError("router weights do not match the block configuration")
        self.register_buffer("router_weight", weights.router.to(device, torch.float32).contiguous())
        self.register_buffer("gate_up_weight", weights.gate_up.to(device, dtype).contiguous())
        self.register_buffer("down_weight", weights.down.to(device, dtype).contiguous())
        self.register_buffer("routing_bias", torch.zeros(self.config.experts, device=device))
        self._workspaces = {}
        self._route_buffers = {}
        self.extension = get_extension()
        if expert_dtype == "fp8_e4m3":
            # gate/up weights in e4m3 with one scale per output channel (weight row);
            # the down GEMM stays bf16
            rows = self.gate_up_weight.shape[0] * self.gate_up_weight.shape[1]
            q = torch.empty(self.gate_up_weight.shape, dtype=torch.float8_e4m3fn, device=device)
            scale = torch.empty(rows, dtype=torch.float32, device=device)
            self.extension.quantize_rows_e4m3(
                self.gate_up_weight.view(rows, -1), q.view(rows, -1), scale)
            self.register_buffer("gate_up_q", q)
            self.register_buffer("gate_up_scale", scale)

    def set_routing_pattern(self, pattern):
        if pattern not in ("balanced", "skewed"):
            raise ValueError("routing pattern must be balanced or skewed")
        self.routing_bias.zero_()
        if pattern == "skewed":
            self.routing_bias[: self.config.topk] = 5.0

    def route(self, x):
        """fp32 logits, top-k with ties to the lower index, softmax of the selected scores."""
        key = (x.shape[0], x.device)
        if key not in self._route_buffers:
            shape = (x.shape[0], self.config.topk)
            self._route_buffers[key] = (
                torch.empty(shape, device=x.device, dtype=torch.int32),
                torch.empty(shape, device=x.device, dtype=torch.int64),
                torch.empty(shape, device=x.device, dtype=torch.float32),
                torch.empty((x.shape[0], self.config.experts), device=x.device, dtype=torch.float32),
            )
        ids32, ids64, weights, logits = self._route_buffers[key]
        self.extension.route_out(
            x, self.router_weight, self.routing_bias, logits, ids32, ids64, weights
        )
        return ids32, ids64, weights

    def logits(self, x):
        """The fp32 router logits of the last route() call for this token count."""
        return self._route_buffers[(x.shape[0], x.device)][3]

    def workspace(self, x):
        key = (x.shape[0], x.dtype, x.device)
        if key not in self._workspaces:
            cfg = self.config
            transport = CudaWorkspace(
                x.shape[0], cfg.hidden, cfg.experts, cfg.topk, x.dtype, device=x.device,
                alignment=cfg.alignment,
            )
            rows = transport.capacity_rows
            projection_rows = rows if self.implementation == "cuda" else 0
            fp8 = self.expert_dtype == "fp8_e4m3"
            self._workspaces[key] = LayerWorkspace(
                transport,
                torch.empty((projection_rows, 2 * cfg.intermediate), device=x.device, dtype=x.dtype),
                torch.empty((rows, cfg.intermediate), device=x.device, dtype=x.dtype),
                torch.empty((rows, cfg.hidden), device=x.device, dtype=x.dtype),
                torch.empty((rows, cfg.hidden), device=x.device, dtype=torch.float8_e4m3fn)
                if fp8 else None,
                torch.empty(rows, device=x.device, dtype=torch.float32) if fp8 else None,
            )
        return self._workspaces[key]

    def experts_forward(self, state):
        transport = state.transport
        ext = self.extension
        if self.expert_dtype == "fp8_e4m3":
            # per-row e4m3 activations, e4m3 gate/up GEMM dequantised in its epilogue
            ext.quantize_rows_e4m3(transport.packed, state.packed_q, state.packed_scale)
            if self.implementation == "cuda_fused":
                ext.grouped_gemm_swiglu_e4m3_out(state.packed_q, state.packed_scale, self.gate_up_q,
                                                 self.gate_up_scale, transport.offsets,
                                                 state.activated)
            else:
                ext.grouped_gemm_e4m3_out(state.packed_q, state.packed_scale, self.gate_up_q,
                                          self.gate_up_scale, transport.offsets, state.projection)
                ext.swiglu_out(state.projection, transport.offsets[-1:], state.activated)
        elif self.implementation == "cuda_fused":
            ext.grouped_gemm_swiglu_out(
                transport.packed, self.gate_up_weight, transport.offsets, state.activated
            )
        else:
            ext.grouped_gemm_out(
                transport.packed, self.gate_up_weight, transport.offsets, state.projection
            )
            ext.swiglu_out(state.projection, transport.offsets[-1:], state.activated)
        ext.grouped_gemm_out(
            state.activated, self.down_weight, transport.offsets, state.expert_output
        )
        return state.expert_output

    @torch.inference_mode()
    def forward(self, x, out=None):
        """Block output for x[T,hidden].  Without `out` the result is the
        workspace's reusable output view; with `out` (a contiguous [T,hidden]
        tensor of x's dtype and device) the combine writes there instead."""
        if x.ndim != 2 or x.shape[1] != self.config.hidden or not x.is_contiguous():
            raise ValueError("expected contiguous x[T,hidden]")
        if x.dtype != self.gate_up_weight.dtype or x.device != self.gate_up_weight.device:
            raise ValueError("input dtype/device must match expert weights")
        check_out(out, x)
        if x.shape[0] == 0:
            return torch.empty_like(x) if out is None else out
        state = self.workspace(x)
        ids32, ids64, weights = self.route(x)
        state.transport.dispatch(x, ids32, ids64)
        output = self.experts_forward(state)
        return state.transport.combine(output, weights, out)
