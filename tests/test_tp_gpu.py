"""Tensor parallelism on 2 GPUs over NCCL: the two-micro-batch forward, whose all-reduces
overlap the other micro-batch's kernels, equals the unsplit TP=2 forward bit for bit (the
per-token arithmetic is the same) and matches the TP=1 forward of the same weights within
the model-level cosine bound (TP sums bf16 partials; TP=1 accumulates in fp32).
Skipped on a machine with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LENGTHS = [1000, 700, 1300, 1000, 1000]   # 5000 tokens: above the overlap threshold


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model_and_batch(dev):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from mes_b200 import synthetic
    from mes_b200.core.gpu_worker import GPUWorker
    from mes_b200.schemas.config import MESConfig
    from mes_b200.ultils.loader import load_weights
    cfg = synthetic.qwen3_0_6b(num_hidden_layers=2)
    worker = GPUWorker(MESConfig(model_config=cfg), device=dev)
    load_weights(worker.model, synthetic.awq_weights(cfg, seed=0, device=dev))
    ids, pos, last = synthetic.packed_batch(LENGTHS, cfg.vocab_size, seed=1)
    return worker, torch.from_numpy(ids).to(dev), torch.from_numpy(pos).to(dev), last


def _worker(rank, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from mes_b200 import _C
    from mes_b200.core.gpu_worker import tp_nccl_environment
    from mes_b200.models.qwen2 import DecoderModel
    tp_nccl_environment(2)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    worker = None
    try:
        worker, ids, pos, last = _model_and_batch(dev)
        with torch.no_grad():
            DecoderModel.overlap_min_tokens = 1 << 30
            unsplit = worker.model(ids, pos).float().cpu()
            DecoderModel.overlap_min_tokens = 4096
            overlapped = worker.model(ids, pos).float().cpu()
        # Bucketed CUDA graphs at tp = 2: each micro-batch is padded to its own bucket (the
        # 5000-token batch splits at 3000: 3000 -> 3072 and 2000 -> 2048 tokens), so the
        # graph's micro-batch boundary is fixed by the bucket; real rows equal the eager
        # forward's.
        from mes_b200 import synthetic
        graphs = []
        for i, lengths in enumerate([LENGTHS, [900, 2100, 1400, 700]]):
            hids, hpos, hlast = synthetic.packed_batch(lengths, worker.model.model.embed_tokens.weight.shape[0], seed=i)
            worker.use_cuda_graphs = True
            got = worker.embed(hids, hpos, hlast).numpy()
            worker.use_cuda_graphs = False
            want = worker.embed(hids, hpos, hlast).numpy()
            graphs.append(bool(np.array_equal(got, want)))
        assert _C.take_device_error() == 0
        if rank == 0:
            q.put((unsplit.numpy(), overlapped.numpy(), np.asarray(last), graphs,
                   worker.captures))
    finally:
        if worker is not None:
            worker.release_graphs()
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_overlapped_forward_matches():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    from test_configs_gpu import get_from_ranks
    unsplit, overlapped, last, graphs, captures = get_from_ranks(q, procs, timeout=600)
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert np.array_equal(unsplit, overlapped)
    assert all(graphs), graphs
    assert captures == 2, captures     # bucket layouts (3072, 2048) and (3072, 2304)

    worker, ids, pos, _ = _model_and_batch(torch.device("cuda", 0))
    with torch.no_grad():
        tp1 = worker.model(ids, pos).float().cpu().numpy()
    a, b = overlapped[last], tp1[last]
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    assert cos.min() >= 0.9995, cos
