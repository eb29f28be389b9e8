"""Tensor-parallel row linear on 2, 4 and 8 GPUs (one process per GPU),
reduced by NCCL and by the peer-memory kernel.

Each rank holds a K-shard of the o_proj / down_proj weight; orin_tp_linear_row
computes its fp32 partial, all-reduces it over NCCL and applies the residual
and the single rounding.  The result must match the unsharded oracle on every
rank.  Column-parallel shards (q/k/v by head, packed gate/up) are plain
orin_linear calls on the shard and are checked the same way."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

H, IM, M = 1024, 2048, 96


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import orininfer_b200 as ob
    from oracle import oracle as orc
    from orininfer_b200 import tp
    from orininfer_b200.synth import seeded
    from tests._util import EXACT_MIN, assert_close, bits, from_bits

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        comm = tp.TPComm(rank, world, rank, tp.exchange_unique_id(rank), timeout_s=60.0)
        act = seeded((M, IM), 1, 1.0)
        wd = seeded((H, IM), 2, 0.02)
        res = seeded((M, H), 3, 1.0)
        # row-parallel down_proj with the residual folded in
        ks = IM // world
        a_dev = act[:, rank * ks:(rank + 1) * ks].contiguous().to(dev)
        w_dev = tp.shard_cols(wd, rank, world).to(dev)
        r_dev = res.to(dev)
        out = comm.linear_row(a_dev, w_dev, residual=r_dev)
        comm.wait()
        ob.device_check()
        ref = orc.linear(bits(act), bits(wd), 0, "residual", bits(res))
        # the fp32 sum over ranks differs from one GPU's only in summation order
        assert_close(out.cpu().float(), from_bits(ref, torch.float16).float(),
                     f"row-parallel rank {rank}", exact_min=EXACT_MIN)

        # the entry point without a caller partial buffer (file-scope device
        # array): the same kernels and summation order, so the same bits
        import ctypes

        from orininfer_b200 import _lib

        def row_static(stream=None):
            o = torch.empty_like(out)
            s = torch.cuda.current_stream() if stream is None else stream
            st = _lib.lib.orin_tp_linear_row_static(
                comm._h, ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(a_dev.data_ptr()),
                ctypes.c_void_p(w_dev.data_ptr()), M, H, ks, 0, ctypes.c_void_p(r_dev.data_ptr()),
                ctypes.c_void_p(s.cuda_stream))
            assert st == _lib.OK, _lib.lib.orin_last_error()
            comm.wait()
            ob.device_check()
            return o

        for _ in range(2):
            assert torch.equal(row_static().view(torch.int16), out.view(torch.int16)), \
                "static scratch vs caller scratch (nccl)"

        # The same calls reduced over NVLink peer memory, summed in rank order:
        # deterministic, within the bar of the oracle, and for two ranks
        # (p0 + p1 either way) the bits of the NCCL path.
        comm.enable_p2p(M * H)
        outs = [comm.linear_row(a_dev, w_dev, residual=r_dev) for _ in range(3)]
        comm.wait()
        ob.device_check()
        assert_close(outs[0].cpu().float(), from_bits(ref, torch.float16).float(),
                     f"p2p row-parallel rank {rank}", exact_min=EXACT_MIN)
        if world == 2:
            assert torch.equal(outs[0].view(torch.int16), out.view(torch.int16)), "p2p vs nccl"
        out = outs[0]
        for i, o in enumerate(outs[1:]):
            assert torch.equal(o.view(torch.int16), out.view(torch.int16)), f"p2p call {i + 1}"
        for _ in range(2):
            assert torch.equal(row_static().view(torch.int16), out.view(torch.int16)), \
                "static scratch vs caller scratch (p2p)"
        # captured once, replayed: the epoch lives in device memory
        static_out = torch.empty_like(out)
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                comm.linear_row(a_dev, w_dev, residual=r_dev, out=static_out, stream=cs)
        torch.cuda.current_stream().wait_stream(cs)
        for rep in range(3):
            static_out.zero_()
            g.replay()
            torch.cuda.synchronize()
            ob.device_check()
            assert torch.equal(static_out.view(torch.int16), out.view(torch.int16)), \
                f"graph replay {rep}"
        del g
        # no residual, and rows that do not split evenly over the ranks
        m7 = 7
        a7 = seeded((m7, IM), 8, 1.0)
        o7 = comm.linear_row(a7[:, rank * ks:(rank + 1) * ks].contiguous().to(dev), w_dev)
        comm.wait()
        ob.device_check()
        ref7 = orc.linear(bits(a7), bits(wd), 0, "none")
        assert_close(o7.cpu().float(), from_bits(ref7, torch.float16).float(),
                     f"p2p no residual M=7 rank {rank}", exact_min=EXACT_MIN)
        # vocabulary-parallel LM head + greedy argmax over ragged shards, with
        # exact ties planted in different shards: 9-bit reversals of residues
        # 1, 2, 257, 88, 487 are 256, 128, 257, 52, 463 -> position 600
        V, Kv = 1000, 512
        hv = seeded((3, Kv), 60, 1.0)
        wv = seeded((V, Kv), 61, 0.02)
        top = (seeded((1, Kv), 62, 1.0).float() * 0.5)[0]
        for m in (0, 2):
            if float(hv[m].float() @ top) < 0:
                hv[m] = -hv[m]
        for pos in (1, 2, 257, 600, 999):
            wv[pos] = top.half()
        lo, hi = tp.ragged_split(V, world)[rank]
        hv_dev = hv.to(dev)
        tok = comm.lm_head_argmax(hv_dev, wv[lo:hi].contiguous().to(dev), lo)
        whole = ob.lm_head_argmax(hv_dev, wv.to(dev))
        comm.wait()
        ob.device_check()
        assert torch.equal(tok, whole), (tok, whole)
        assert int(tok[0]) == 600 and int(tok[2]) == 600, tok

        # column-parallel gate/up with SwiGLU on this rank's packed shard
        wg = seeded((IM, H), 4, 0.02)
        wu = seeded((IM, H), 5, 0.02)
        x = seeded((M, H), 6, 1.0)
        y = ob.linear(x.to(dev), tp.shard_gate_up(wg.to(dev), wu.to(dev), rank, world),
                      epilogue="swiglu")
        ob.device_check()
        ims = IM // world
        g, u = tp.shard_gate_up_rows(wg, wu, rank, world)
        ref2 = orc.linear(bits(x), orc.pack_gate_up(bits(g), bits(u)), 0, "swiglu")
        assert_close(y.cpu().float(), from_bits(ref2, torch.float16).float(),
                     f"column-parallel rank {rank}", exact_min=EXACT_MIN)
        assert y.shape == (M, ims)
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report, never hang the parent
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_and_column_parallel(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, msg = q.get(timeout=300)
        results[r] = msg
    for p in procs:
        p.join(timeout=120)
    assert all(m == "ok" for m in results.values()), results
