"""Tensor-parallel Q4Linear on 2+ GPUs of one box (one process per GPU).

Row-parallel shards summed by the library's NVLink all-reduce
(sf_q4_linear_allreduce) and by NCCL must both match the unsharded oracle
(normwise 1e-3 for the fp32 GEMV, 5e-3 when T reaches the bf16 prefill GEMM),
every rank must hold bitwise the same Y from the peer all-reduce, and
alternating exchange slots must stay correct over repeated calls.  A rank
that does not join a call makes the other rank's bounded wait expire with
SF_ERR_TIMEOUT instead of hanging, and poisons the communicator: the ranks
that join late, and every later call on any rank, get SF_ERR_COMM and no
value.  NVLS is off (NCCL_NVLS_ENABLE=0) and the
peer kernel uses plain peer loads/stores.  Skipped with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    out = {"rank": rank}
    try:
        from oracle import q4_oracle as O
        from siliconfer_b200 import _lib, quant as Q
        from siliconfer_b200.tensor_parallel import ColumnParallelQ4Linear, PeerComm, RowParallelQ4Linear
        comm = PeerComm(slot_bytes=8 << 20, arena_bytes=64 << 20)
        errs, same = [], []
        for case, (n, k, t, asym, xdt) in enumerate([(512, 2048, 1, False, torch.float32),
                                                     (1024, 4096, 4, True, torch.float16),
                                                     (256, 1024, 64, False, torch.bfloat16),
                                                     (384, 3072, 2, True, torch.float32)]):
            rng = np.random.default_rng(100 + case)
            w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
            p, s, z = Q.pack_weights_asym(w, 128) if asym else (*Q.pack_weights_sym(w, 128), None)
            bias = rng.normal(0, 0.1, n).astype(np.float32)
            peer = RowParallelQ4Linear(p, s, z, bias, 128, rank=rank, world=world, device=dev, comm=comm)
            nccl = RowParallelQ4Linear(p, s, z, bias, 128, rank=rank, world=world, device=dev, mode="nccl")
            col = ColumnParallelQ4Linear(p, s, z, bias, 128, rank=rank, world=world, device=dev)
            k0, k1 = peer.k_range
            for rep in range(3):
                x = rng.normal(0, 1, (t, k)).astype(np.float32)
                xd = torch.from_numpy(x).to(dev).to(xdt)
                xq = xd.float().cpu().numpy()
                ref = O.gemm(p, s, z, xq, 128) + bias
                tol = 5e-3 if t >= 48 else 1e-3
                ya = peer(xd[:, k0:k1].contiguous())
                yb = nccl(xd[:, k0:k1].contiguous())
                yc = col(xd)
                torch.cuda.synchronize()
                lo, hi = col.rows
                errs.append((case, rep, O.normwise_rel_err(ya.cpu().numpy(), ref),
                             O.normwise_rel_err(yb.cpu().numpy(), ref),
                             O.normwise_rel_err(yc.cpu().numpy(), ref[:, lo:hi]), tol))
                g = [torch.empty_like(ya) for _ in range(world)]
                dist.all_gather(g, ya)
                same.append(all(torch.equal(g[0], gi) for gi in g))
        out["errs"], out["same"] = errs, same
        # the fused step: two layers of 7 projections, all-reduces inside one launch,
        # checked against the unfused step (local GEMV + NCCL) on the same inputs
        from siliconfer_b200.tensor_parallel import TPStepRunner
        from siliconfer_b200.q4_linear import Q4Linear
        H, F = 512, 1536
        shapes = [(H, H), (128, H), (128, H), (H, H), (F, H), (F, H), (H, F)]
        layers = []
        for li in range(2):
            lay = []
            for pi, (n, k) in enumerate(shapes):
                rng = np.random.default_rng(1000 * li + pi)
                w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
                pq, sq = Q.pack_weights_sym(w, 128)
                if pi in (3, 6):
                    from siliconfer_b200.tensor_parallel import shard_row
                    pq, sq, _, _ = shard_row(pq, sq, None, 128, rank, world)
                else:
                    from siliconfer_b200.tensor_parallel import shard_column
                    pq, sq, _, _ = shard_column(pq, sq, None, rank, world)
                lay.append(Q4Linear(pq, sq, group_size=128, device=dev))
            layers.append(lay)
        fused = TPStepRunner(layers, tokens=2, mode="fused", comm=comm, device=dev)
        ref = TPStepRunner(layers, tokens=2, mode="nccl", device=dev)
        g = torch.Generator(device=dev).manual_seed(5)
        fused.x.copy_(torch.randn(fused.x.shape, generator=g, device=dev).to(fused.x.dtype))
        ref.x.copy_(fused.x)
        fused.capture()
        ref.capture()
        fe = []
        for rep in range(4):
            fused.run()
            ref.run()
            torch.cuda.synchronize()
            a, b = fused.red.double(), ref.red.double()
            fe.append(((a - b).abs().max() / b.abs().max()).item())
        out["fused_err"] = fe
        gg = [torch.empty_like(fused.red) for _ in range(world)]
        dist.all_gather(gg, fused.red)
        out["fused_same"] = all(torch.equal(gg[0], x) for x in gg)
        # the same step in the decoder's order (each phase waits for the one before)
        ordered = TPStepRunner(layers, tokens=2, mode="fused", comm=comm, device=dev, ordered=True)
        ordered.x.copy_(fused.x)
        ordered.capture()
        oe = []
        for rep in range(3):
            ordered.run()
            torch.cuda.synchronize()
            a, b = ordered.red.double(), ref.red.double()
            oe.append(((a - b).abs().max() / b.abs().max()).item())
        out["ordered_err"] = oe
        del fused, ref, ordered
        out["dev_err_ok"] = _lib.load().sf_q4_check_device_error()
        # bounded wait: rank 0 starts an all-reduce that no other rank joins
        dist.barrier()
        lib = _lib.load()
        buf = torch.full((256,), float(rank + 1), device=dev)
        res = torch.full((256,), -1.0, device=dev)

        def allreduce():
            _lib.check(lib.sf_tp_allreduce(comm.comm, buf.data_ptr(), res.data_ptr(), 0, None, 256, 256,
                                           torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            return lib.sf_q4_check_device_error()

        if rank == 0:
            out["timeout_status"] = allreduce()
            out["after"] = lib.sf_q4_check_device_error()
        dist.barrier()
        # the others join late: they must get an error, not a value
        if rank != 0:
            out["late_status"] = allreduce()
            out["late_untouched"] = bool((res == -1.0).all().item())
        dist.barrier()
        # and the communicator stays poisoned on every rank
        out["again_status"] = allreduce()
        dist.barrier()
        comm.close()
    except Exception as exc:  # reported to the parent
        import traceback
        out["exc"] = traceback.format_exc()
    q.put(out)
    dist.destroy_process_group()


def test_row_parallel_peer_and_nccl_match_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda d: d["rank"])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert "exc" not in r, r["exc"]
        assert r["dev_err_ok"] == 0
        assert all(r["same"]), "ranks disagree on the peer all-reduce result"
        for case, rep, ea, eb, ec, tol in r["errs"]:
            assert ea <= tol and eb <= tol and ec <= tol, (r["rank"], case, rep, ea, eb, ec)
    for r in res:
        assert max(r["fused_err"]) <= 1e-5, r["fused_err"]
        assert max(r["ordered_err"]) <= 1e-5, r["ordered_err"]
        assert r["fused_same"]
    assert res[0]["timeout_status"] == 7        # SF_ERR_TIMEOUT
    assert res[0]["after"] == 0                 # the error word was read and cleared
    for r in res[1:]:
        assert r["late_status"] == 8, r         # SF_ERR_COMM: a late rank gets no value
        assert r["late_untouched"], "a late rank's output was written from a stale exchange"
    for r in res:
        assert r["again_status"] == 8, r        # poisoned until the communicator is made again
