"""Split-KV decode on 2 GPUs (skipped with fewer): each rank keeps only its
own pages of K/V and its k_bar rows; the combined output of
SplitKVDecode.step must match one GPU decoding the whole sequence.  Both
exchange paths: NCCL all-gathers, and the library's peer-memory exchange
(PeerBackend: plain stores into the peers' IPC-mapped regions + bounded flag
waits), eagerly and replayed from a captured CUDA graph.  NVLS is off."""

import datetime
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

RP = dict(block_size=64, local_blocks=8, topk=8, topm=16, idx_scale=128 / math.sqrt(128), floor=1e-4, sigma=1.0)
NBLK, BS, H, D, DI = 2048, 64, 10, 128, 128


def _problem():
    g = torch.Generator().manual_seed(21)
    k = (torch.randn(NBLK, BS, H, D, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(NBLK, BS, H, D, generator=g) * 0.5).to(torch.bfloat16)
    kbar = torch.randn(1, NBLK, DI, generator=g)
    q = (torch.randn(2, H, D, generator=g) * 0.5).to(torch.bfloat16)
    iq = torch.randn(2, DI, generator=g).to(torch.bfloat16)
    return k, v, kbar, q, iq


def _worker(rank, world, port, result_q, exchange="nccl"):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from srswa import ops
        from srswa.split_kv import SplitKVDecode
        k, v, kbar, q, iq = _problem()
        S = NBLK * BS - 5
        q_pos = torch.tensor([S - 2, S - 1], device=dev, dtype=torch.int64)
        backend = None
        if exchange != "nccl":   # p2p-<mode>: the peer-memory exchange
            from srswa.split_kv import PeerBackend
            backend = PeerBackend(rows=2, topm=RP["topm"], heads=H, head_dim=D, mode=exchange[4:])
        dec = SplitKVDecode(nblk_total=NBLK, nblk_filled=NBLK, sm_scale=1 / math.sqrt(D), rank=rank, world=world,
                            backend=backend, **RP)
        lo, hi = dec.plan.lo, dec.plan.hi
        table = torch.zeros(1, NBLK, dtype=torch.int32, device=dev)
        table[0, lo:hi] = torch.arange(hi - lo, dtype=torch.int32, device=dev)
        layer = dict(kbar=kbar[:, lo:hi].contiguous().to(dev), k_cache=k[lo:hi].to(dev), v_cache=v[lo:hi].to(dev),
                     block_table=table)
        qd, iqd = q.to(dev), iq.to(dev)
        outs = [dec.step(qd, iqd, q_pos, layer, p_range=(S - 2, S - 1), out_dtype=torch.float32).clone()
                for _ in range(2)]          # two steps: the exchange epochs advance
        if exchange != "nccl":
            # captured once, replayed: the epochs advance on the device
            s_ = torch.cuda.Stream()
            s_.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s_):
                with torch.cuda.graph(graph):
                    g_out = dec.step(qd, iqd, q_pos, layer, p_range=(S - 2, S - 1), out_dtype=torch.float32)
            torch.cuda.current_stream().wait_stream(s_)
            for _ in range(3):
                graph.replay()
                outs.append(g_out.clone())
            torch.cuda.synchronize()
            dec.backend.check()
            del graph
        out = outs[0]
        if rank == 0:
            full_t = torch.arange(NBLK, dtype=torch.int32, device=dev)[None]
            sel = ops.route(iq.to(dev), kbar.to(dev), q_pos=q_pos, rows_per_seq=2, want=("topi32", "bias"), **RP)
            ref = torch.empty(2, H, D, device=dev)
            ops.decode_attend(q.to(dev), k.to(dev), v.to(dev), sel["topi32"], sel["bias"], block_size=BS,
                              local_blocks=RP["local_blocks"], sm_scale=1 / math.sqrt(D), out=ref,
                              block_table=full_t, q_pos=q_pos, rows_per_req=2)
            torch.cuda.synchronize()
            result_q.put(("ok", max(float((o - ref).abs().max()) for o in outs)))
        torch.cuda.synchronize()
        if exchange != "nccl":
            dec.backend.close()
        dist.barrier()
    except Exception as e:
        result_q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "p2p-ll", "p2p-flag", "p2p-launch"])
def test_split_kv_two_gpus_matches_one_gpu(exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(2, port, q, exchange), nprocs=2, join=True, start_method="spawn")
    msg = q.get(timeout=60)
    assert msg[0] == "ok", msg
    assert msg[1] < 1e-5
