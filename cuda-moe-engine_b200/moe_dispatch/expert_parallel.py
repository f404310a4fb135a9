"""Expert-parallel MoE block over torch.distributed (one process per GPU).

The reference is single-GPU (README.md:161-163); this module adds the
expert-parallel layer the north star asks for.  Rank r of P owns experts
[r*E/P, (r+1)*E/P) and its own slice of the tokens.  One forward:

  1. route the local tokens over all E experts           (moe_route)
  2. pack them by global expert, compact                 (moe_dispatch, alignment 1)
     -- destination ranks own contiguous expert ranges, so the packed rows are
        already grouped by destination rank
  3. exchange per-(rank, expert) counts                  (all_to_all_single)
  4. exchange the rows                                   (all_to_all_single, uneven splits)
  5. regroup received rows into expert-major spans       (moe_ep_layout, moe_ep_regroup)
  6. gate/up GEMM + SwiGLU, down GEMM on local experts   (tcgen05 grouped GEMMs)
  7. put the outputs back in received order              (moe_ep_regroup)
  8. return them to their source ranks                   (all_to_all_single)
  9. weighted combine at the source                      (moe_combine)

Inside an expert, received rows are ordered by source rank, and ranks hold
consecutive token ranges, so the grouped rows are exactly the rows a single GPU
would pack: the output is bit-identical to MoEBlock on one GPU.

Steps 3-4 need the split sizes on the host, so a forward synchronises once
after the count exchange; the count, split and row-exchange helpers take any
process group and tensors on any device (the gloo tests run them on CPU).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .layer import MoEConfig
from .workspace import CudaWorkspace, capacity_rows
from ._extension import get_extension


def expert_range(experts, ranks, rank):
    """Experts owned by `rank`: [first, first + per_rank)."""
    if experts % ranks:
        raise ValueError(f"{experts} experts do not split evenly over {ranks} ranks")
    per_rank = experts // ranks
    return rank * per_rank, per_rank


def exchange_counts(counts, ranks, group=None):
    """counts[E] (this rank's rows per global expert) -> recv[P, E_l]: rows each
    source rank sends for each of this rank's experts."""
    experts = counts.numel()
    local = experts // ranks
    recv = torch.empty(ranks * local, dtype=counts.dtype, device=counts.device)
    dist.all_to_all_single(recv, counts.contiguous(), group=group)
    return recv.view(ranks, local)


def split_sizes(counts, recv_counts, ranks):
    """Host split sizes: rows sent to each rank, rows received from each rank."""
    send = counts.view(ranks, -1).sum(dim=1).tolist()
    recv = recv_counts.sum(dim=1).tolist()
    return [int(v) for v in send], [int(v) for v in recv]


def exchange_rows(send, send_rows, recv, recv_rows, group=None):
    """Rows to their destinations: send[sum(send_rows), H] -> recv[sum(recv_rows), H]."""
    dist.all_to_all_single(recv, send, output_split_sizes=recv_rows,
                           input_split_sizes=send_rows, group=group)
    return recv


class _Buffers:
    """Device buffers that grow to the largest step seen (no per-step allocation once warm)."""

    def __init__(self):
        self.tensors = {}

    def get(self, name, rows, cols, dtype, device):
        t = self.tensors.get(name)
        if t is None or t.shape[0] < rows or t.shape[1] != cols or t.dtype != dtype:
            t = torch.empty(max(rows, 1), cols, dtype=dtype, device=device)
            self.tensors[name] = t
        return t


class ExpertParallelMoEBlock(torch.nn.Module):
    """MoE block whose experts are sharded over the ranks of `group`.

    router_weight [E, H] fp32 and routing_bias [E] are replicated; gate_up
    [E_l, 2I, H] and down [E_l, H, I] are this rank's experts.  forward(x) takes
    this rank's tokens x [T_l, H] bf16 and returns their outputs [T_l, H].
    """

    def __init__(self, config, router_weight, gate_up, down, *, group=None, device="cuda",
                 routing_bias=None):
        super().__init__()
        self.config = config if isinstance(config, MoEConfig) else MoEConfig(*config)
        self.group = group
        self.ranks = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.first_expert, self.local_experts = expert_range(self.config.experts, self.ranks,
                                                             self.rank)
        device = torch.device(device)
        cfg = self.config
        if tuple(router_weight.shape) != (cfg.experts, cfg.hidden):
            raise ValueError("router weights do not match the block configuration")
        if tuple(gate_up.shape) != (self.local_experts, 2 * cfg.intermediate, cfg.hidden):
            raise ValueError("gate_up must hold this rank's experts [E_l, 2I, H]")
        if tuple(down.shape) != (self.local_experts, cfg.hidden, cfg.intermediate):
            raise ValueError("down must hold this rank's experts [E_l, H, I]")
        self.register_buffer("router_weight", router_weight.to(device, torch.float32).contiguous())
        self.register_buffer("gate_up_weight", gate_up.to(device, torch.bfloat16).contiguous())
        self.register_buffer("down_weight", down.to(device, torch.bfloat16).contiguous())
        bias = torch.zeros(cfg.experts) if routing_bias is None else routing_bias
        self.register_buffer("routing_bias", bias.to(device, torch.float32).contiguous())
        self.extension = get_extension()
        self._transport = {}
        self._route = {}
        self._rows = _Buffers()
        self.last_split_sizes = None

    def _state(self, x):
        key = (x.shape[0], x.device)
        if key not in self._transport:
            cfg = self.config
            self._transport[key] = CudaWorkspace(x.shape[0], cfg.hidden, cfg.experts, cfg.topk,
                                                 x.dtype, device=x.device, alignment=1)
            shape = (x.shape[0], cfg.topk)
            self._route[key] = (
                torch.empty(shape, device=x.device, dtype=torch.int32),
                torch.empty(shape, device=x.device, dtype=torch.int64),
                torch.empty(shape, device=x.device, dtype=torch.float32),
                torch.empty((x.shape[0], cfg.experts), device=x.device, dtype=torch.float32),
            )
            e_l = self.local_experts
            self._layout = (
                torch.empty(self.ranks, e_l, dtype=torch.int32, device=x.device),
                torch.empty(self.ranks, e_l, dtype=torch.int32, device=x.device),
                torch.empty(e_l + 1, dtype=torch.int32, device=x.device),
            )
        return self._transport[key], self._route[key]

    @torch.inference_mode()
    def forward(self, x, events=None):
        """`events`, if given, maps stage names ("exchange", "gemm1", "gemm2",
        "return") to (start, end) CUDA events recorded around those stages."""
        cfg = self.config

        def mark(name, which):
            if events is not None and name in events:
                events[name][which].record()

        if x.ndim != 2 or x.shape[1] != cfg.hidden or not x.is_contiguous():
            raise ValueError("expected contiguous x[T,hidden]")
        if x.dtype != torch.bfloat16 or x.device != self.gate_up_weight.device:
            raise ValueError("input must be bf16 on the block's device")
        ext = self.extension
        transport, (ids32, ids64, weights, logits) = self._state(x)
        tokens = x.shape[0]
        n = tokens * cfg.topk
        if tokens:
            ext.route_out(x, self.router_weight, self.routing_bias, logits, ids32, ids64, weights)
        transport.dispatch(x, ids32, ids64)
        recv_counts = exchange_counts(transport.counts, self.ranks, self.group)
        send_rows, recv_rows = split_sizes(transport.counts, recv_counts, self.ranks)
        self.last_split_sizes = (send_rows, recv_rows)
        n_recv = sum(recv_rows)
        grouped_rows = capacity_rows(n_recv, self.local_experts, 1, cfg.alignment)
        bufs = self._rows
        recv = bufs.get("recv", n_recv, cfg.hidden, x.dtype, x.device)
        grouped = bufs.get("grouped", grouped_rows, cfg.hidden, x.dtype, x.device)
        activated = bufs.get("activated", grouped_rows, cfg.intermediate, x.dtype, x.device)
        expert_out = bufs.get("expert_out", grouped_rows, cfg.hidden, x.dtype, x.device)
        back = bufs.get("back", n, cfg.hidden, x.dtype, x.device)
        mark("exchange", 0)
        exchange_rows(transport.packed[:n], send_rows, recv[:n_recv], recv_rows, self.group)
        mark("exchange", 1)
        src_start, dst_start, offsets = self._layout
        ext.ep_layout(recv_counts, cfg.alignment, src_start, dst_start, offsets)
        ext.ep_regroup(recv, grouped, recv_counts, src_start, dst_start, offsets, n_recv, True)
        mark("gemm1", 0)
        ext.grouped_gemm_swiglu_out(grouped, self.gate_up_weight, offsets, activated)
        mark("gemm1", 1)
        mark("gemm2", 0)
        ext.grouped_gemm_out(activated, self.down_weight, offsets, expert_out)
        mark("gemm2", 1)
        ext.ep_regroup(expert_out, recv, recv_counts, src_start, dst_start, offsets, n_recv, False)
        mark("return", 0)
        exchange_rows(recv[:n_recv], recv_rows, back[:n], send_rows, self.group)
        mark("return", 1)
        if tokens:
            transport.combine(back[:n], weights)
        return transport.output
