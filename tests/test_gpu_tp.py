"""Row-parallel quantized linear on 2, 4 and 8 GPUs (one process each, NCCL for set-up
and the comparison path only), against the unsharded CPU oracle and against the NCCL
all-reduce comparison path: up to three tokens run the GEMV with the all-reduce fused
into its epilogue, four or more the tensor-core GEMM followed by the library's two-shot
all-reduce kernel, which is also checked on its own (rtd_tp_allreduce).

Each world size is skipped when the box has fewer GPUs.  NVLS is switched off and the kernel's peer
traffic is plain stores, so a rank that leaves early cannot fault the others; the
timeout case makes one rank skip a call and checks that the other finishes with
RTD_ERR_PEER_TIMEOUT instead of waiting.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL_EXACT = 2e-5


def _rel(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    import oracle
    from runtimed_b200 import _lib, synth
    from runtimed_b200.errors import ConfigError
    from runtimed_b200.tp import RowParallelLinear, TpComm
    from runtimed_b200.weights import Context

    OUT_TOL = {torch.float32: RTOL_EXACT, torch.float16: 1e-3, torch.bfloat16: 4e-3}
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    out = {}
    try:
        ctx = Context.for_device(dev)
        comm = TpComm(ctx, rank, world, max_n=4096)
        shapes = [(12, 4096, 256 * world), (14, 1000, 256 * world), (8, 2056, 64 * world)]
        for t, n, k in shapes:
            raw = synth.quant_matrix(t, n, k, seed=5, stream=t)
            bias = np.random.default_rng(t).normal(0, 0.02, n).astype(np.float32)
            rpl = RowParallelLinear.from_full_weight(raw, t, n, k, bias, rank, world, comm=comm, device=dev)
            ks = k // world
            # M <= 3: the fused GEMV (f32 rows at M = 3: two launches, two epochs in one
            # call); M >= 4: the GEMM and the two-shot all-reduce (M = 130: two chunks)
            for call, (m, dt) in enumerate([(1, torch.bfloat16), (3, torch.float32), (4, torch.float16),
                                            (6, torch.float32), (64, torch.bfloat16), (130, torch.float32),
                                            (1, torch.bfloat16)]):
                x = synth.activations(m, k, seed=100 * t + call)
                xt = torch.from_numpy(x).to(dt)
                want = oracle.qgemv_f64(t, raw, n, k, xt.float().numpy()) + bias[None, :]
                xs = xt[:, rank * ks:(rank + 1) * ks].contiguous().to(dev)
                y = rpl.forward(xs).float()
                yn = rpl.forward_nccl(xs).float()
                torch.cuda.synchronize()
                ctx.check_device_status()
                gathered = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(gathered, y)
                # y comes back in x's dtype: its rounding bounds the error (bf16 ~2^-9 RMS)
                tol = OUT_TOL[dt]
                rf, rn = _rel(y.cpu().numpy(), want), _rel(yn.cpu().numpy(), want)
                # four or more tokens run the tensor-core GEMM (f16-rounded weights, 1e-3
                # gate) on both paths
                tol = tol if m <= 3 else max(tol, 1e-3)
                out[(t, call)] = (rf <= tol, rn <= tol, all(bool(torch.equal(g, gathered[0])) for g in gathered),
                                  rf, rn)
        # the stand-alone two-shot all-reduce: sum of every rank's f32 partial + bias once
        for call, (m, n, dt) in enumerate([(1, 4096, torch.float32), (7, 1000, torch.bfloat16),
                                           (128, 4096, torch.float32), (300, 33, torch.float16)]):
            parts = [torch.from_numpy(synth.activations(m, n, seed=700 + call, stream=q)) for q in range(world)]
            bias = torch.from_numpy(np.random.default_rng(call).normal(0, 0.5, n).astype(np.float32))
            want = sum(p.double() for p in parts) + bias.double()
            y = comm.allreduce(parts[rank].to(dev), bias=bias.to(dev), out_dtype=dt).float()
            torch.cuda.synchronize()
            ctx.check_device_status()
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            r = _rel(y.cpu().numpy(), want.numpy())
            out[("ar", call)] = (r <= OUT_TOL[dt], True, all(bool(torch.equal(g, gathered[0])) for g in gathered),
                                 r, 0.0)
        # the fused call captured in a CUDA graph: the epoch lives on the device, so
        # every replay exchanges fresh partials (new x each replay, checked each time)
        # (one fused GEMV launch at M = 2, the GEMM + all-reduce at M = 8 in the same graph)
        t, n, k = 14, 1000, 256 * world
        raw = synth.quant_matrix(t, n, k, seed=6, stream=t)
        rpl = RowParallelLinear.from_full_weight(raw, t, n, k, None, rank, world, comm=comm, device=dev)
        ks = k // world
        xs = torch.zeros((2, ks), dtype=torch.float32, device=dev)
        xb = torch.zeros((8, ks), dtype=torch.float32, device=dev)
        rpl.forward(xs)
        rpl.forward(xb)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yg = rpl.forward(xs)
            yb = rpl.forward(xb)
        graph_ok = []
        for rep in range(3):
            x = synth.activations(2, k, seed=900 + rep)
            x8 = synth.activations(8, k, seed=950 + rep)
            xs.copy_(torch.from_numpy(x[:, rank * ks:(rank + 1) * ks]).to(dev))
            xb.copy_(torch.from_numpy(x8[:, rank * ks:(rank + 1) * ks]).to(dev))
            g.replay()
            torch.cuda.synchronize()
            ctx.check_device_status()
            graph_ok.append(_rel(yg.cpu().numpy(), oracle.qgemv_f64(t, raw, n, k, x)) <= RTOL_EXACT)
            graph_ok.append(_rel(yb.cpu().numpy(), oracle.qgemv_f64(t, raw, n, k, x8)) <= 1e-3)
        del g
        out["graph"] = all(graph_ok)
        # only rank 0 makes a call: it finishes with RTD_ERR_PEER_TIMEOUT instead of waiting
        raw = synth.quant_matrix(12, 16, 256 * world, seed=1)
        rpl = RowParallelLinear.from_full_weight(raw, 12, 16, 256 * world, None, rank, world, comm=comm, device=dev)
        dist.barrier()
        timed_out = None
        if rank == 0:
            xs = torch.zeros((1, 256), dtype=torch.bfloat16, device=dev)
            rpl.forward(xs)
            torch.cuda.synchronize()
            try:
                ctx.check_device_status()
                timed_out = False
            except ConfigError as e:
                timed_out = f"status {_lib.RTD_ERR_PEER_TIMEOUT}" in str(e)
        dist.barrier()
        out["timeout"] = timed_out
        comm.close()
    except BaseException as e:  # reported to the parent, which fails the test with it
        out["error"] = f"{type(e).__name__}: {e}"
    finally:
        try:
            dist.destroy_process_group()
        finally:
            q.put((rank, out))  # always: a rank that raised must not leave the parent waiting


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_parallel_fused_allreduce(world):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, out in res.items():
        assert "error" not in out, (rank, out.get("error"))
        assert out["graph"] is True, (rank, "graph replay")
        for key, (fused_ok, nccl_ok, same, rf, rn) in ((k, v) for k, v in out.items() if k not in ("timeout", "graph", "error")):
            assert fused_ok, (rank, key, "fused", rf)
            assert nccl_ok, (rank, key, "nccl", rn)
            assert same, (rank, key, "ranks differ")
    assert res[0]["timeout"] is True


def _model_rank_main(rank, world, port, path, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    from runtimed_b200.qwen2 import Qwen2Model, Session
    from runtimed_b200.tp import TpComm
    from runtimed_b200.weights import Context

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    out = {}
    try:
        comm = TpComm(Context.for_device(dev), rank, world, max_n=4096)
        prompt = list(np.random.default_rng(3).integers(0, 1000, 24))
        for exact in (True, False):  # exact: fused GEMV exchange; else a 24-token GEMM + all-reduce prefill
            model = Qwen2Model(path, device=dev, max_ctx=128, kv_dtype=torch.float32, exact_linears=exact, comm=comm)
            ids, per = Session(model).greedy(prompt, 8)
            per = torch.stack(per)
            gathered = [torch.empty_like(per) for _ in range(world)]
            dist.all_gather(gathered, per)
            res = {"ids": ids, "same": all(bool(torch.equal(g, gathered[0])) for g in gathered)}
            if rank == 0:
                single = Qwen2Model(path, device=dev, max_ctx=128, kv_dtype=torch.float32, exact_linears=exact)
                ids1, per1 = Session(single).greedy(prompt, 8)
                res["ids1"] = ids1
                res["rel"] = [_rel(a.cpu().numpy(), b.cpu().numpy()) for a, b in zip(per, per1)]
                del single
            out[exact] = res
            del model
            torch.cuda.synchronize()
            dist.barrier()
        comm.close()
    except BaseException as e:  # reported to the parent, which fails the test with it
        out["error"] = f"{type(e).__name__}: {e}"
    finally:
        try:
            dist.destroy_process_group()
        finally:
            q.put((rank, out))


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_decoder(world, tmp_path):
    # the Qwen2 decoder split over `world` GPUs (heads and FFN rows column-parallel,
    # attn_output / ffn_down row-parallel through rtd_tp_qlinear_row) gives the logits and
    # greedy ids of the single-GPU decoder, bit-identical on every rank
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from runtimed_b200 import fixtures

    shape = fixtures.Qwen2Shape(hidden=512, n_layer=2, n_head=8, n_kv=4, ffn=1024, vocab=1000,
                                formats={k: 8 for k in fixtures.DEFAULT_FORMATS})
    path = str(tmp_path / "tp.gguf")
    fixtures.write_qwen2_gguf(path, shape, seed=4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_model_rank_main, args=(r, world, port, path, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, out in res.items():
        assert "error" not in out, (rank, out.get("error"))
        for exact in (True, False):
            assert out[exact]["same"], (rank, exact, "ranks differ")
            assert out[exact]["ids"] == res[0][exact]["ids"]
    for exact, tol in ((True, 1e-5), (False, 3e-3)):
        r0 = res[0][exact]
        assert r0["ids"] == r0["ids1"], exact
        assert max(r0["rel"]) <= tol, (exact, r0["rel"])
