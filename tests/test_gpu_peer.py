"""GPU checks of the all-gather fused into the GEMM epilogue
(tc_cuda_qlinear_gather) and of the device flag barrier (tc_cuda_peer_barrier).

On one GPU the "peer" replicas are other buffers of the same device: every
kernel family (pair GEMM with TMA stores and with plain stores, one-CTA GEMM,
GEMV, dense weights) must write each output into this rank's Y and into every
replica, inside this rank's column range only.  The barrier is checked with one
rank (it must pass) and with a flag that no rank ever raises (it must give up
after its time limit, set TC_STATUS_TIMEOUT and return).  The two-process test
runs the real thing across GPUs when at least two are visible.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

PATHS = {"gemv": (5, 0, "f32", 1e-5), "one_cta": (100, 3, "bf16", 1e-4), "pair": (300, 0, "bf16", 1e-4)}


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("out_dtype", [0, 2])
@pytest.mark.parametrize("epilogue", [False, True])
def test_replicas_receive_every_output(ctx, where, out_dtype, epilogue):
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    n, k, n_total, col = 300, 768, 1024, 256          # this rank's columns [256, 556) of 1024
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=1))
    w = tcc.Weight.upload(ctx, 12, n, k, raw)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=2)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    tdt = tcc._torch_dtype(out_dtype)
    sentinel = 7.0
    ys = [torch.full((m, n_total), sentinel, device="cuda", dtype=tdt) for _ in range(3)]
    item = ys[0].element_size()
    bias = torch.randn(n, device="cuda") if epilogue else None
    ctx.set_path(path)
    try:
        tcc.qlinear(ctx, w, x, out=ys[0][:, col:col + n], out_dtype=out_dtype, bias=bias,
                    activation="gelu_tanh" if epilogue else None,
                    peers=[ys[1].data_ptr() + col * item, ys[2].data_ptr() + col * item])
    finally:
        ctx.set_path(0)
    assert ctx.status() == 0
    ref = oracle.qlinear_ref(xb, raw, 12, n, k, staging)
    if epilogue:
        ref = oracle.epilogue_ref(ref, bias=bias.cpu().numpy(), activation="gelu_tanh")
    bound = f32b if out_dtype == 0 else 3e-3
    for y in ys:
        h = y.float().cpu().numpy()
        assert oracle.rel_l2(h[:, col:col + n], ref) <= bound
        assert np.all(h[:, :col] == sentinel) and np.all(h[:, col + n:] == sentinel)
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("out_dtype", [0, 2])
def test_swiglu_replicas_receive_every_output(ctx, where, out_dtype):
    """A SwiGLU weight (one output per gate / up row pair) with N-column
    replicas: this rank's 320 outputs [256, 576) of 1024 land in Y and in both
    replicas, nothing outside that range is touched (the pair kernel's
    16-output TMA boxes included)."""
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    f, k, n_total, col = 320, 768, 1024, 256
    rg = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=31))
    ru = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=32))
    w = tcc.Weight.upload_glu(ctx, 12, f, k, rg, ru)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=33)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    tdt = tcc._torch_dtype(out_dtype)
    sentinel = 7.0
    ys = [torch.full((m, n_total), sentinel, device="cuda", dtype=tdt) for _ in range(3)]
    item = ys[0].element_size()
    bias = np.random.default_rng(34).standard_normal(2 * f).astype(np.float32) * 0.5
    ctx.set_path(path)
    try:
        tcc.qlinear(ctx, w, x, out=ys[0][:, col:col + f], out_dtype=out_dtype, bias=torch.from_numpy(bias).cuda(),
                    peers=[ys[1].data_ptr() + col * item, ys[2].data_ptr() + col * item])
    finally:
        ctx.set_path(0)
    assert ctx.status() == 0
    acc = np.concatenate([oracle.qlinear_ref(xb, rg, 12, f, k, staging), oracle.qlinear_ref(xb, ru, 12, f, k, staging)],
                         axis=1)
    ref = oracle.epilogue_ref(acc, bias=bias, glu=True)
    bound = f32b if out_dtype == 0 else 3e-3
    for y in ys:
        h = y.float().cpu().numpy()
        assert oracle.rel_l2(h[:, col:col + f], ref) <= bound
        assert np.all(h[:, :col] == sentinel) and np.all(h[:, col + f:] == sentinel)
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


def test_dense_weight_replicas(ctx):
    import torch
    from turbocider_b200 import cuda as tcc
    n, k, m = 64, 96, 40
    w32 = np.random.default_rng(3).standard_normal((n, k)).astype(np.float32)
    w = tcc.Weight.upload(ctx, 0, n, k, w32.tobytes())
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    ys = [torch.zeros(m, 2 * n, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    tcc.qlinear(ctx, w, x, out=ys[0][:, n:], peers=[ys[1].data_ptr() + n * 2])
    assert ctx.status() == 0
    assert torch.equal(ys[0], ys[1]) and not ys[0][:, :n].any()


@pytest.mark.parametrize("engine", [("copy", 0), ("copy", 2), ("kernel", 3), ("kernel", 148)],
                         ids=["copy", "copy-fanout2", "kernel-3", "kernel-148"])
@pytest.mark.parametrize("layout", ["shard_major", "strided"])
def test_copy_engine_push_fills_every_replica(ctx, layout, engine):
    """tc_cuda_peer_push: this rank's shard of a GEMM output reaches the same
    place in every replica (linear copies for a shard-major Y[g][M][N/g], 2-D
    copies for column shards of Y[M, N]) by the copy engines (back to back or
    fanned out) or by the SMs' push kernel (few or many blocks); nothing
    outside the shard is written."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k, m, world, rank = 256, 512, 300, 3, 1
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=4))
    w = tcc.Weight.upload(ctx, 12, n, k, raw)
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    if layout == "shard_major":
        ys = [torch.zeros(world, m, n, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
        shard = ys[0][rank]
        src, width, rows, pitch = shard.data_ptr(), m * n * 2, 1, m * n * 2
        offset = rank * m * n * 2
    else:
        ys = [torch.zeros(m, world * n, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
        shard = ys[0][:, rank * n:(rank + 1) * n]
        src, width, rows, pitch = shard.data_ptr(), n * 2, m, world * n * 2
        offset = rank * n * 2
    tcc.qlinear(ctx, w, x, out=shard)
    dst = (C.c_void_p * (world - 1))(*[ys[i].data_ptr() + offset for i in range(1, world)])
    kind, n_par = engine
    if kind == "copy":
        ctx.set_push_fanout(n_par)
    else:
        ctx.set_push_kernel(n_par)
    try:
        for _ in range(2):
            tcc._check(tcc.lib().tc_cuda_peer_push(ctx.handle, C.c_void_p(src), dst, world - 1, width, rows, pitch,
                                                   pitch, None))
    finally:
        ctx.set_push_fanout(0)
        ctx.set_push_kernel(0)
    torch.cuda.synchronize()
    assert ctx.status() == 0
    assert shard.abs().sum() > 0
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    total = sum(int((y != 0).sum()) for y in ys)
    assert total == world * int((shard != 0).sum())


def _flags(n):
    import torch
    return torch.zeros(n, dtype=torch.int32, device="cuda")


def test_barrier_one_rank(ctx):
    import torch
    from turbocider_b200 import cuda as tcc
    f = _flags(1)
    arr = (C.c_void_p * 1)(f.data_ptr())
    for epoch in (1, 2, 3):
        tcc._check(tcc.lib().tc_cuda_peer_barrier(ctx.handle, arr, 1, 0, epoch, 100000, None))
        torch.cuda.synchronize()
        assert int(f[0]) == epoch
    assert ctx.status() == 0


def test_barrier_gives_up_on_a_missing_rank(ctx):
    """Rank 1 never arrives: the wait ends after its limit with
    TC_STATUS_TIMEOUT, and the device stays usable."""
    import torch
    from turbocider_b200 import cuda as tcc
    mine, other = _flags(2), _flags(2)
    arr = (C.c_void_p * 2)(mine.data_ptr(), other.data_ptr())
    tcc._check(tcc.lib().tc_cuda_peer_barrier(ctx.handle, arr, 2, 0, 1, 20000, None))
    torch.cuda.synchronize()
    assert ctx.status() & tcc.STATUS_TIMEOUT
    assert int(other[0]) == 1 and int(mine[0]) == 1 and int(mine[1]) == 0
    assert float(torch.ones(4, device="cuda").sum()) == 4.0
    assert ctx.status() == 0


def _two_rank_worker(rank, world, port, q, mode="fused"):
    import datetime
    import sys
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from turbocider_b200 import cuda as tcc
    from turbocider_b200 import shard
    from turbocider_b200.peer import PeerGroup
    try:
        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        ctx = tcc.Context(rank)
        if mode == "kernel":
            ctx.set_push_kernel(64)
        n, k, m = 1024, 1024, 520
        raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=9))
        per = shard.rows_per_rank(n, world)
        b, rows = shard.shard_rows(n, world, rank)
        w = tcc.Weight.upload(ctx, 12, n, k, raw, n_begin=b, n_count=rows)
        xb = kq_cases.synthetic_x_bf16(m, k, seed=10)
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        pg = PeerGroup(ctx, timeout_us=5_000_000)
        buf = pg.alloc(m * world * per * 2)
        if mode == "fused":
            y = buf.tensor((m, world * per), torch.bfloat16)
            for rep in range(3):
                tcc.qlinear(ctx, w, x, out=y[:, rank * per:rank * per + rows], peers=pg.peers_of(buf, rank * per * 2))
                pg.barrier()
            torch.cuda.synchronize()
            got = y.float().cpu().numpy()[:, :n]
        else:
            # copy-engine gather (bench.py's default): the GEMM writes this
            # rank's slot of a shard-major Y[world][M][per]; a side stream
            # pushes the slot to every peer, then the flag barrier
            y = buf.tensor((world, m, per), torch.bfloat16)
            side = torch.cuda.Stream()
            for rep in range(3):
                y[rank].zero_()
                tcc.qlinear(ctx, w, x, out=y[rank][:, :rows])
                done = torch.cuda.Event()
                done.record()
                side.wait_event(done)
                pg.push(buf, rank * m * per * 2, m * per * 2, stream=side)
                pg.barrier(side)
                torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            got = shard.assemble(y.float().cpu().numpy(), n)
        status = ctx.status()
        err = oracle.rel_l2(got, oracle.qlinear_ref(xb, raw, 12, n, k, "bf16"))
        del y
        pg.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, status, err))
    except Exception as e:  # reported to the parent
        q.put((rank, -1, repr(e)))


@pytest.mark.parametrize("mode", ["fused", "copy", "kernel"])
def test_two_rank_gather(mode):
    """Two ranks on two GPUs: each computes its column shard and the full Y on
    each rank matches the oracle, with the all-gather fused into the GEMM
    epilogue, pushed by the copy engines, or pushed by the SMs' kernel."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    port = 29500 + os.getpid() % 1000 + {"fused": 0, "copy": 7, "kernel": 13}[mode]
    procs = [ctx_mp.Process(target=_two_rank_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, err in res:
        assert status == 0, (rank, err)
        assert err <= 3e-3, (rank, err)
