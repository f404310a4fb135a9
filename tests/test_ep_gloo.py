"""Expert-parallel exchange protocol on CPU ranks (gloo, world size 2).

Each rank routes, dispatches and computes its experts with the CPU oracle, and
exchanges counts and rows with the module's own helpers
(exchange_counts, split_sizes, exchange_rows); the layout is the oracle's
restatement of moe_ep_layout.  The gathered outputs must equal the
single-process oracle block bit for bit.  A second test kills one rank before
the exchange and checks that the survivor's collective fails within the
process-group timeout instead of hanging.
"""

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout=60):
    for path in (ROOT / "cuda-moe-engine_b200", ROOT, ROOT / "tests" / "golden"):
        sys.path.insert(0, str(path))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout))


def _ep_worker(rank, world, port, result_dir):
    _setup(rank, world, port)
    import cases
    from moe_dispatch.expert_parallel import exchange_counts, exchange_rows, expert_range, split_sizes
    from oracle import moe_oracle as oracle

    spec = {"config": (64, 32, 8, 2), "weight_seed": 4, "x_seed": 5, "tokens": 48,
            "bias": "skewed", "name": "ep"}
    hidden, inter, experts, topk = spec["config"]
    router, gate_up, down = cases.block_weights(spec)
    bias = cases.block_bias(spec)
    x_all = cases.block_input(spec)
    per_rank = spec["tokens"] // world
    x = x_all[rank * per_rank:(rank + 1) * per_rank].contiguous()
    first, local = expert_range(experts, world, rank)

    _, ids32, _, weights = oracle.route(x, router, bias, topk)
    counts, offsets, slots, inverse, packed = oracle.dispatch(x, ids32, experts, 1)
    recv_counts = exchange_counts(counts, world)
    send_rows, recv_rows = split_sizes(counts, recv_counts, world)
    recv = torch.empty(sum(recv_rows), hidden, dtype=x.dtype)
    exchange_rows(packed, send_rows, recv, recv_rows)
    layout = oracle.ep_layout(recv_counts, 8)
    grouped = oracle.ep_regroup(recv, recv_counts, layout)
    grouped = torch.nan_to_num(grouped)
    gu = gate_up[first:first + local].contiguous()
    dn = down[first:first + local].contiguous()
    act = oracle.swiglu(oracle.grouped_gemm(grouped, gu, layout[2]), int(layout[2][-1]))
    eo = oracle.grouped_gemm(act, dn, layout[2])
    eo_recv = oracle.ep_regroup(eo, recv_counts, layout, grouping=False)
    back = torch.empty(packed.shape[0], hidden, dtype=x.dtype)
    exchange_rows(eo_recv, recv_rows, back, send_rows)
    out = oracle.combine(back, inverse, weights)
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    if rank == 0:
        torch.save({"ep": torch.cat(gathered), "sends": send_rows}, Path(result_dir) / "ep.pt")
    dist.destroy_process_group()


def test_two_rank_exchange_matches_single_process(tmp_path):
    mp.spawn(_ep_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases
    from oracle import moe_oracle as oracle

    spec = {"config": (64, 32, 8, 2), "weight_seed": 4, "x_seed": 5, "tokens": 48,
            "bias": "skewed", "name": "ep"}
    router, gate_up, down = cases.block_weights(spec)
    single = oracle.block_forward(cases.block_input(spec), router, cases.block_bias(spec),
                                  gate_up, down, 2)["output"]
    result = torch.load(tmp_path / "ep.pt", weights_only=True)
    assert torch.equal(result["ep"], single)
    assert sum(result["sends"]) == 24 * 2


def _dead_rank_worker(rank, world, port, result_dir):
    _setup(rank, world, port, timeout=5)
    from moe_dispatch.expert_parallel import exchange_counts

    if rank == 1:
        os._exit(0)  # leaves between steps, before the count exchange
    try:
        exchange_counts(torch.zeros(8, dtype=torch.int32), world)
        outcome = "completed"
    except Exception as error:  # the collective must fail, not hang
        outcome = type(error).__name__
    (Path(result_dir) / "outcome.txt").write_text(outcome)
    os._exit(0)


def test_a_departed_rank_is_detected_by_the_collective_timeout(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung after its peer left")
    outcome = (tmp_path / "outcome.txt").read_text()
    assert outcome != "completed"
