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

Each grouped row is computed on its own (GEMM rows are independent), so the
output is bit-identical to MoEBlock on one GPU whatever the order of the rows
inside an expert: source-major on the NCCL path (ranks hold consecutive token
ranges, so these are the rows a single GPU would pack), arrival order on the
P2P path.

Two exchange backends:

* ``"p2p"`` (default, up to 8 ranks on one node): every rank shares one
  region of its HBM with the others through CUDA IPC.  Counts go out with peer
  stores and flags, senders write rows straight into the owners' expert-major
  buffers and owners write results straight back into the sources' packed
  slots (``moe_ep_p2p``); the down GEMM returns the rows itself
  (``moe_ep_p2p_down_return``).  Optionally the exchange runs beside the
  gate/up GEMM, which then takes each expert's tiles in the order their rows
  arrive (``moe_ep_p2p_gate_up``, ``overlap=True``).  No host
  synchronisation: the whole step can be captured in a CUDA graph.  Waits on peers are bounded and report through
  ``moe_device_status``.
* ``"nccl"``: steps 3-4 and 8 as ``all_to_all_single`` with the split sizes
  read on the host (one synchronisation per forward), and the regroup kernels.
  The count, split and row-exchange helpers take any process group and tensors
  on any device (the gloo tests run them on CPU).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .layer import MoEConfig, check_out
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


class _DeviceArray:
    """A raw device allocation seen as an array (for torch.as_tensor, zero copy)."""

    def __init__(self, address, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(address), False), "version": 3,
                                         "strides": None}


class PeerExchange:
    """This rank's P2P exchange region (shared over CUDA IPC), the peers' regions
    mapped into this process, and the rank-local step state."""

    def __init__(self, lib, group, ranks, rank, experts, hidden, grouped_rows, back_rows,
                 device):
        self.lib, self.ranks, self.rank = lib, ranks, rank
        self.shape = (experts, hidden, grouped_rows, back_rows)
        nbytes = lib.moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows)
        if nbytes < 0:
            raise ValueError("expert-parallel P2P needs <= 8 ranks, experts divisible by ranks")
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        self._check(lib.moe_peer_alloc(nbytes, ctypes.addressof(own), ctypes.addressof(handle)))
        self.own = own.value
        handles = [None] * ranks
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened, bases = [], []
        for r in range(ranks):
            if r == rank:
                bases.append(self.own)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(handles[r])
            self._check(lib.moe_peer_open(ctypes.addressof(buf), ctypes.addressof(peer)))
            self.opened.append(peer.value)
            bases.append(peer.value)
        self.regions = (ctypes.c_void_p * ranks)(*bases)
        words = lib.moe_ep_p2p_state_words(ranks, experts)
        self.state = torch.zeros(words, dtype=torch.int32, device=device)
        g_off = lib.moe_ep_p2p_region_offset(ranks, experts, hidden, grouped_rows, back_rows, 0)
        b_off = lib.moe_ep_p2p_region_offset(ranks, experts, hidden, grouped_rows, back_rows, 1)
        self.grouped = torch.as_tensor(
            _DeviceArray(self.own + g_off, (grouped_rows, hidden), "<i2"), device=device
        ).view(torch.bfloat16)
        self.back = torch.as_tensor(
            _DeviceArray(self.own + b_off, (back_rows, hidden), "<i2"), device=device
        ).view(torch.bfloat16)
        local = experts // ranks
        self.offsets = self.state[4 + experts: 4 + experts + local + 1]
        dist.barrier(group=group)

    def _check(self, status):
        if status != 0:
            raise RuntimeError(self.lib.moe_last_error().decode())

    def close(self):
        """Unmap the peers' regions and free this rank's (after the device is idle)."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        self.grouped = self.back = None
        for ptr in self.opened:
            self.lib.moe_peer_close(ptr)
        self.lib.moe_peer_free(self.own)
        self.own, self.opened = None, []


class _Lane:
    """One micro-batch's buffers on the P2P path: transport workspace, route
    outputs, exchange region, GEMM rows and (after the first) its own stream."""

    def __init__(self):
        self.transport = {}
        self.route = {}
        self.exchange = None
        self.rows = _Buffers()
        self.stream = None


class ExpertParallelMoEBlock(torch.nn.Module):
    """MoE block whose experts are sharded over the ranks of `group`.

    router_weight [E, H] fp32 and routing_bias [E] are replicated; gate_up
    [E_l, 2I, H] and down [E_l, H, I] are this rank's experts.  forward(x) takes
    this rank's tokens x [T_l, H] bf16 and returns their outputs [T_l, H].

    fused_return=True (p2p only; the default there) runs the down GEMM with an
    epilogue that stores each result row straight into its source rank's slot
    (moe_ep_p2p_down_return) instead of a separate return copy, so the return
    crosses NVLink while the GEMM runs.  With the CTA-pair tile the epilogue
    stages each 32 x 32 chunk in shared memory and stores 64-byte row
    segments.  Measured on two B200s: the return stage falls from 2.19 to
    0.40 ms at the E=256 configuration and from 0.157 to 0.080 ms at the
    Mixtral shape, the down GEMM slows by 0.14 and 0.015 ms.

    overlap=True (p2p with micro_batches=1) overlaps the row exchange with the
    gate/up GEMM: this rank's own rows are copied first, the other ranks' rows
    go out on a second stream, and the GEMM (moe_ep_p2p_gate_up) takes each
    expert's tiles in the order their rows arrive, waiting on a peer's rows
    flag before a tile that needs them.  Inside an expert the grouped rows
    follow that arrival order; GEMM rows are independent, so the output bits
    do not change.  It is off by default: on two B200s it measured slower
    than the serial exchange (Mixtral shape 2.26-2.28 against 2.21 ms per
    step, E=256 13.96-19.46 against 13.87 ms).  Tiles taken group by group
    stream each expert's weights once per group, the send kernel beside the
    GEMM slows it, and on fewer SMs the send itself slows (85-330 GB/s).

    micro_batches=m (p2p only) splits the local tokens into m consecutive
    slices, each with its own exchange region, run on their own streams in a
    pipeline: slice i sends its rows once slice i-1's rows have arrived (so the
    copy runs under slice i-1's gate/up GEMM), and starts its GEMMs once slice
    i-1's down GEMM is done (so slice i-1's results travel back under them).
    Every rank must use the same m.  GEMM rows are computed independently, so
    the output bits do not depend on m.
    """

    def __init__(self, config, router_weight, gate_up, down, *, group=None, device="cuda",
                 routing_bias=None, backend=None, timeout_ms=10000, fused_return=None,
                 micro_batches=1, overlap=None):
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
        if backend is None:
            backend = "p2p" if self.ranks <= 8 else "nccl"
        if backend not in ("p2p", "nccl"):
            raise ValueError("backend must be p2p or nccl")
        self.backend = backend
        self.timeout_ms = int(timeout_ms)
        if fused_return is None:
            fused_return = backend == "p2p"
        if fused_return and backend != "p2p":
            raise ValueError("fused_return needs the p2p backend")
        self.fused_return = bool(fused_return)
        self.micro_batches = int(micro_batches)
        if self.micro_batches < 1 or (self.micro_batches > 1 and backend != "p2p"):
            raise ValueError("micro_batches must be 1, or >= 1 with the p2p backend")
        if overlap is None:
            overlap = False
        if overlap and (backend != "p2p" or self.micro_batches != 1):
            raise ValueError("overlap needs the p2p backend and micro_batches=1")
        self.overlap = bool(overlap)
        self._lanes = [_Lane() for _ in range(self.micro_batches)]
        self._outputs = {}
        self._last_key = None
        self._last_keys = []

    @property
    def exchange(self):
        """The first micro-batch's P2P exchange (None before the first p2p forward)."""
        return self._lanes[0].exchange if self.backend == "p2p" else None

    def last_send_counts(self, lane=None):
        """Rows this rank's last forward packed for each global expert (device int32
        [E]), over all micro-batches or for micro-batch `lane` only."""
        if self.backend != "p2p":
            return self._transport[self._last_key].counts
        picked = range(len(self._last_keys)) if lane is None else [lane]
        total = None
        for i in picked:
            c = self._lanes[i].transport[self._last_keys[i]].counts
            total = c.clone() if total is None else total + c
        return total

    def last_grouped_rows(self, lane=None):
        """Grouped rows this rank's experts received in the last p2p forward, over all
        micro-batches or for micro-batch `lane` only (synchronises)."""
        e, e_l = self.config.experts, self.local_experts
        picked = self._lanes if lane is None else [self._lanes[lane]]
        return sum(int(ln.exchange.state[4 + e + e_l].item()) for ln in picked)

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
        self._last_key = key
        return self._transport[key], self._route[key]

    def _lane_state(self, lane, x):
        key = (x.shape[0], x.device)
        if key not in lane.transport:
            cfg = self.config
            lane.transport[key] = CudaWorkspace(x.shape[0], cfg.hidden, cfg.experts, cfg.topk,
                                                x.dtype, device=x.device, alignment=1)
            shape = (x.shape[0], cfg.topk)
            lane.route[key] = (
                torch.empty(shape, device=x.device, dtype=torch.int32),
                torch.empty(shape, device=x.device, dtype=torch.int64),
                torch.empty(shape, device=x.device, dtype=torch.float32),
                torch.empty((x.shape[0], cfg.experts), device=x.device, dtype=torch.float32),
            )
        return key, lane.transport[key], lane.route[key]

    @torch.inference_mode()
    def forward(self, x, events=None, out=None):
        """`events`, if given, maps stage names ("exchange", "gemm1", "gemm2",
        "return", and with overlap "send": the other ranks' rows, on the side
        stream) to (start, end) CUDA events recorded around those stages.
        `out`, if given, receives the combined rows instead of the workspace's
        reusable output view."""
        cfg = self.config

        def mark(name, which):
            if events is not None and name in events:
                events[name][which].record()

        if x.ndim != 2 or x.shape[1] != cfg.hidden or not x.is_contiguous():
            raise ValueError("expected contiguous x[T,hidden]")
        if x.dtype != torch.bfloat16 or x.device != self.gate_up_weight.device:
            raise ValueError("input must be bf16 on the block's device")
        check_out(out, x)
        if self.backend == "p2p":
            return self._forward_p2p(x, mark, out)
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
            return transport.combine(back[:n], weights, out)
        return transport.output if out is None else out

    def _peer_exchange(self, lane, tokens, device):
        """The lane's exchange region, (re)created for `tokens` local tokens; a
        collective over the group (every rank calls it in the same order)."""
        cfg = self.config
        grouped_rows = capacity_rows(self.ranks * tokens * min(cfg.topk, self.local_experts),
                                     self.local_experts, 1, cfg.alignment)
        back_rows = max(tokens * cfg.topk, 1)
        shape = (cfg.experts, cfg.hidden, grouped_rows, back_rows)
        if lane.exchange is not None and lane.exchange.shape == shape:
            return lane.exchange
        if lane.exchange is not None:
            lane.exchange.close()
        lane.exchange = PeerExchange(self.extension.lib, self.group, self.ranks, self.rank,
                                     cfg.experts, cfg.hidden, grouped_rows, back_rows, device)
        return lane.exchange

    def _p2p(self, op, rows, aux, ex=None):
        ex = self.exchange if ex is None else ex
        experts, hidden, grouped_rows, back_rows = ex.shape
        self.extension._call(
            ex.state.device, self.extension.lib.moe_ep_p2p, op,
            None if rows is None else rows.data_ptr(), None if aux is None else aux.data_ptr(),
            ctypes.addressof(ex.regions), ex.state.data_ptr(), self.ranks, self.rank, experts,
            self.config.alignment, hidden, grouped_rows, back_rows, self.timeout_ms,
        )

    def _forward_p2p(self, x, mark, out=None):
        """Steps 1-9 over peer memory: no host synchronisation (graph-capturable).
        With micro_batches > 1 the slices run as the pipeline described in the
        class docstring; `mark` events cover the first slice only."""
        tokens = x.shape[0]
        m = self.micro_batches
        if m == 1:
            result, _, _, key = self._lane_forward(self._lanes[0], x, mark, out)
            self._last_keys = [key]
            return result
        if out is None:
            key = (tokens, x.device)
            if key not in self._outputs:
                self._outputs[key] = torch.empty_like(x)
            out = self._outputs[key]
        bounds = [tokens * i // m for i in range(m + 1)]
        main = torch.cuda.current_stream(x.device)
        start = torch.cuda.Event()
        start.record(main)
        received = gemm_done = None
        finished, keys = [], []
        for i, lane in enumerate(self._lanes):
            if i > 0 and lane.stream is None:
                lane.stream = torch.cuda.Stream(device=x.device)
            stream = main if i == 0 else lane.stream
            with torch.cuda.stream(stream):
                if i > 0:
                    stream.wait_event(start)
                _, received, gemm_done, key = self._lane_forward(
                    lane, x[bounds[i]:bounds[i + 1]], mark if i == 0 else None,
                    out[bounds[i]:bounds[i + 1]], after_received=received, after_gemm=gemm_done)
                keys.append(key)
                if i > 0:
                    done = torch.cuda.Event()
                    done.record(stream)
                    finished.append(done)
        for done in finished:
            main.wait_event(done)
        self._last_keys = keys
        return out

    def _lane_forward(self, lane, x, mark=None, out=None, after_received=None, after_gemm=None):
        """One slice on the current stream.  Returns (output, event after its rows
        arrived, event after its down GEMM, workspace key)."""
        cfg = self.config
        ext = self.extension
        mark = mark or (lambda name, which: None)
        stream = torch.cuda.current_stream(x.device)
        key, transport, (ids32, ids64, weights, logits) = self._lane_state(lane, x)
        tokens = x.shape[0]
        n = tokens * cfg.topk
        if tokens:
            ext.route_out(x, self.router_weight, self.routing_bias, logits, ids32, ids64, weights)
        transport.dispatch(x, ids32, ids64)
        ex = self._peer_exchange(lane, tokens, x.device)
        rows = ex.grouped.shape[0]
        activated = lane.rows.get("activated", rows, cfg.intermediate, x.dtype, x.device)
        expert_out = lane.rows.get("expert_out", rows, cfg.hidden, x.dtype, x.device)
        self._p2p(0, None, transport.counts, ex)
        if after_received is not None:
            stream.wait_event(after_received)
        sent = None
        if self.overlap:
            # other ranks' rows on the side stream, beside this rank's GEMM
            if lane.stream is None:
                lane.stream = torch.cuda.Stream(device=x.device)
            counted = torch.cuda.Event()
            counted.record(stream)
            lane.stream.wait_event(counted)
            with torch.cuda.stream(lane.stream):
                mark("send", 0)
                self._p2p(6, transport.packed, transport.offsets, ex)
                mark("send", 1)
                sent = torch.cuda.Event()
                sent.record(lane.stream)
            mark("exchange", 0)
            self._p2p(5, transport.packed, transport.offsets, ex)
            mark("exchange", 1)
        else:
            mark("exchange", 0)
            self._p2p(1, transport.packed, transport.offsets, ex)
            self._p2p(2, None, None, ex)
            mark("exchange", 1)
        received = torch.cuda.Event()
        received.record(stream)
        if after_gemm is not None:
            stream.wait_event(after_gemm)
        mark("gemm1", 0)
        if self.overlap:
            experts, hidden, grouped_rows, back_rows = ex.shape
            ext._call(ex.state.device, ext.lib.moe_ep_p2p_gate_up, self.gate_up_weight.data_ptr(),
                      activated.data_ptr(), ctypes.addressof(ex.regions), ex.state.data_ptr(),
                      self.ranks, self.rank, experts, hidden, cfg.intermediate, grouped_rows,
                      back_rows, self.timeout_ms)
        else:
            ext.grouped_gemm_swiglu_out(ex.grouped, self.gate_up_weight, ex.offsets, activated)
        mark("gemm1", 1)
        mark("gemm2", 0)
        if self.fused_return:
            # down GEMM whose epilogue writes each result row into its source's slot
            experts, hidden, grouped_rows, back_rows = ex.shape
            ext._call(ex.state.device, ext.lib.moe_ep_p2p_down_return, activated.data_ptr(),
                      self.down_weight.data_ptr(), ctypes.addressof(ex.regions),
                      ex.state.data_ptr(), self.ranks, self.rank, experts, hidden,
                      cfg.intermediate, grouped_rows, back_rows)
            mark("gemm2", 1)
            gemm_done = torch.cuda.Event()
            gemm_done.record(stream)
            mark("return", 0)
        else:
            ext.grouped_gemm_out(activated, self.down_weight, ex.offsets, expert_out)
            mark("gemm2", 1)
            gemm_done = torch.cuda.Event()
            gemm_done.record(stream)
            mark("return", 0)
            self._p2p(3, expert_out, None, ex)
        self._p2p(4, None, None, ex)
        mark("return", 1)
        if sent is not None:
            stream.wait_event(sent)
        if tokens:
            result = transport.combine(ex.back[:n], weights, out)
        else:
            result = transport.output if out is None else out
        return result, received, gemm_done, key

    def close(self):
        """Release the P2P exchange regions (call on every rank, before the process group ends)."""
        for lane in self._lanes:
            if lane.exchange is not None:
                lane.exchange.close()
                lane.exchange = None
