"""Token sharding across ranks, checked on CPU with gloo (world size 2).

The mHC path shards by token: each rank runs its own tokens with no collective
in the forward pass, and only the parameter gradients are summed across ranks
(DDP / NCCL in training).  These tests run two gloo ranks as child processes
and check, with the oracle, that

* the sharded forward equals the single-process forward on the concatenated
  tokens, row for row;
* all-reduced (summed) parameter gradients equal the full-batch gradients;
* the timing reduction used by ``bench.py`` (max over ranks) picks the slowest
  rank;
* ``bench.py``'s gradient all-reduce handles a parameter with no gradient on
  one rank, and its bucketed all-reduce (launched from gradient hooks during
  backward) equals the flat one.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mhc_oracle as O

N, C, T_PER_RANK, WORLD = 4, 64, 24, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params():
    gen = torch.Generator().manual_seed(0)
    return O.make_full_params(N, C, init="bench", generator=gen)


def _inputs(rank):
    gen = torch.Generator().manual_seed(100 + rank)
    return torch.randn(1, T_PER_RANK, N * C, generator=gen)


def _loss(p, x):
    out = O.full_forward(x, p, lambda z: z * 0.5, N, C, sinkhorn_iters=20)
    return out, (out.float() ** 2).mean() * out.numel()


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        p = _params()
        leaves = [p.phi_weight, p.alpha_pre, p.bias_pre, p.alpha_post, p.bias_post, p.alpha_res, p.bias_res]
        for t in leaves:
            t.requires_grad_(True)
        out, loss = _loss(p, _inputs(rank))
        loss.backward()
        gs = [t.grad.clone() for t in leaves]
        for g in gs:
            dist.all_reduce(g, op=dist.ReduceOp.SUM)
        # bench.py reduces the step time with a max over ranks
        t = torch.tensor([1.0 + rank])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # numpy copies pickle by value (tensors would be shared through file
        # descriptors that vanish when this process exits)
        q.put((rank, out.detach().numpy().copy(), [g.numpy().copy() for g in gs], t.item()))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def sharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in range(WORLD):
        r, out, gs, tmax = q.get(timeout=300)
        res[r] = (torch.from_numpy(out), [torch.from_numpy(g) for g in gs], tmax)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    return res


def test_sharded_forward_matches_single_process(sharded):
    p = _params()
    x = torch.cat([_inputs(r) for r in range(WORLD)], dim=1)
    with torch.no_grad():
        full, _ = _loss(p, x)
    for r in range(WORLD):
        shard = full[:, r * T_PER_RANK:(r + 1) * T_PER_RANK]
        assert torch.allclose(sharded[r][0], shard, rtol=1e-6, atol=1e-6)


def test_allreduced_grads_equal_full_batch_grads(sharded):
    p = _params()
    leaves = [p.phi_weight, p.alpha_pre, p.bias_pre, p.alpha_post, p.bias_post, p.alpha_res, p.bias_res]
    for t in leaves:
        t.requires_grad_(True)
    x = torch.cat([_inputs(r) for r in range(WORLD)], dim=1)
    _, loss = _loss(p, x)
    loss.backward()
    for r in range(WORLD):
        for g_shard, t in zip(sharded[r][1], leaves):
            assert torch.allclose(g_shard, t.grad, rtol=1e-4, atol=1e-5)


def test_step_time_is_max_over_ranks(sharded):
    assert all(sharded[r][2] == float(WORLD) for r in range(WORLD))


def _grad_worker(rank, port, q):
    """bench.py's gradient all-reduce with a parameter that got no gradient on
    one rank (an MoE expert no token of that rank was routed to)."""
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        ps = [torch.nn.Parameter(torch.zeros(5)), torch.nn.Parameter(torch.zeros(3, 2, dtype=torch.bfloat16)),
              torch.nn.Parameter(torch.zeros(4, dtype=torch.bfloat16))]
        ps[0].grad = torch.full((5,), 1.0 + rank)
        ps[1].grad = torch.full((3, 2), 2.0 * (rank + 1), dtype=torch.bfloat16)
        if rank == 0:
            ps[2].grad = torch.full((4,), 6.0, dtype=torch.bfloat16)  # rank 1 leaves this one None
        bench.allreduce_grads(ps, WORLD)
        t = torch.tensor([1.0])
        dist.all_reduce(t)  # the collective sequence is still aligned
        q.put((rank, [p.grad.float().numpy().copy() for p in ps], t.item()))
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_with_a_missing_gradient():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, port, q)) for r in range(WORLD)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in range(WORLD):
        r, gs, tsum = q.get(timeout=300)
        res[r] = (gs, tsum)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for r in range(WORLD):
        gs, tsum = res[r]
        assert tsum == float(WORLD)
        assert torch.allclose(torch.from_numpy(gs[0]), torch.full((5,), 1.5))
        assert torch.allclose(torch.from_numpy(gs[1]), torch.full((3, 2), 3.0))
        assert torch.allclose(torch.from_numpy(gs[2]), torch.full((4,), 3.0))  # (6 + 0) / 2


def _bucket_worker(rank, port, q):
    """bench.py's overlapped bucketed all-reduce against its flat all-reduce:
    mixed fp32/bf16 parameters, many small buckets, an expert that gets no
    gradient on rank 1, two steps (the views into the flat buffers must stay
    attached across zero())."""
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)

    def make():
        torch.manual_seed(0)
        m = torch.nn.ModuleDict({"a": torch.nn.Linear(8, 16), "b": torch.nn.Linear(16, 16),
                                 "e0": torch.nn.Linear(16, 4, bias=False), "e1": torch.nn.Linear(16, 4, bias=False)})
        m["b"].to(torch.bfloat16)
        return m

    def loss_of(m, x):
        h = torch.tanh(m["a"](x))
        h = m["b"](h.bfloat16()).float()
        y = m["e0"](h)
        if rank == 0:  # rank 1 routes nothing to expert 1
            y = y + m["e1"](h)
        return (y ** 2).mean()

    try:
        ref, buck = make(), make()
        rp, bp = list(ref.parameters()), list(buck.parameters())
        gb = bench.GradBuckets(bp, WORLD, bucket_mb=200 / (1 << 20))
        assert len(gb.buckets) >= 4
        out = []
        for step in range(2):
            gen = torch.Generator().manual_seed(10 * step + rank)
            x = torch.randn(6, 8, generator=gen)
            loss_of(ref, x).backward()
            bench.allreduce_grads(rp, WORLD)
            loss_of(buck, x).backward()
            gb.finish()
            out.append([(a.grad.float().clone(), b.grad.float().clone()) for a, b in zip(rp, bp)])
            assert all(p.grad.data_ptr() >= gb.flat[p.dtype].data_ptr() for p in bp)
            for p in rp:
                p.grad = None
            gb.zero()
        t = torch.tensor([1.0])
        dist.all_reduce(t)
        q.put((rank, [[(a.numpy(), b.numpy()) for a, b in s] for s in out], t.item()))
    finally:
        dist.destroy_process_group()


def test_bucketed_allreduce_equals_flat_allreduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, port, q)) for r in range(WORLD)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in range(WORLD):
        r, steps, tsum = q.get(timeout=300)
        res[r] = (steps, tsum)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for r in range(WORLD):
        steps, tsum = res[r]
        assert tsum == float(WORLD)
        for pairs in steps:
            for a, b in pairs:
                assert torch.equal(torch.from_numpy(a), torch.from_numpy(b))
    # both ranks hold the same averaged gradients
    for (a0, _), (a1, _) in zip(res[0][0][1], res[1][0][1]):
        assert torch.equal(torch.from_numpy(a0), torch.from_numpy(a1))
