"""Parity at the benchmark configurations, against fixtures written by running the
reference's own model code on the CPU (``tests/golden/make_golden.py``).

Each fixture holds, for one configuration's seeded AWQ checkpoint (codes and zero-points
uniform in [0, 15], fp16 scales uniform in [0.002, 0.02]) and batch:
  * ``emb_fp32``: the reference's forward in fp32 on the exactly dequantised weights - the
    "fp32 dequantised reference" the embeddings are compared with;
  * ``emb_bf16``: the reference's forward in bf16 (its deployment dtype) on the same
    weights - its own distance from fp32 is the yardstick for ours;
  * checksums of every checkpoint tensor, so the test proves it regenerated the same
    checkpoint (seeded CPU generator) before comparing.

The weight distribution gives every quantisation group a mean offset (7.5 - z) * s, so
activations and attention logits grow large with depth and every bf16 rounding matters:
against fp32, the reference's own bf16 path reaches a cosine of only 0.994 (worst row) on
the 28-layer 0.6B model and 0.80 on the 28-layer Qwen2-1.5B model (no q/k norm, logits in
the hundreds), but 0.99987 on two 8B-shaped layers.  The bound is therefore relative to
the reference's own deployment path: ours (bf16 kernels, fp32 residual stream) must be on
average at least as close to the fp32 reference as the reference's bf16 path
(mean of 1 - cosine), and its worst row no worse than min(the reference's worst row,
0.9995); where the reference's bf16 path is within 0.9995 everywhere, ours must be too.
"""
import os
import sys

import numpy as np
import pytest
import torch

# Spawned tensor-parallel ranks import this module by name before anything else has loaded
# the package directory as ``mes_b200``.
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()

from mes_b200 import _C, synthetic  # noqa: E402
from mes_b200.core.gpu_worker import GPUWorker
from mes_b200.schemas.config import MESConfig
from mes_b200.ultils.loader import load_weights

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

ARCH = {"c2": (synthetic.qwen3_0_6b, {}),
        "c4_slice": (synthetic.qwen3_8b, dict(num_hidden_layers=2)),
        "c5": (synthetic.qwen2_1_5b, {})}


def _cos(a, b):
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def _checksums(weights: dict) -> dict:
    out = {}
    for name in sorted(weights):
        t = weights[name]
        if t.dtype in (torch.float16, torch.bfloat16):
            t = t.view(torch.int16)
        out[name] = int(t.to(torch.int64).sum())
    return out


def load_config(name):
    """(cfg, weights, lengths, fixture) with the checkpoint regenerated and verified."""
    f = np.load(os.path.join(HERE, "golden", f"ref_awq_{name}.npz"))
    arch, over = ARCH[name]
    cfg = arch(**over)
    weights = synthetic.awq_weights(cfg, seed=int(f["weight_seed"]), device="cpu",
                                    norm_noise=float(f["norm_noise"]))
    sums = _checksums(weights)
    want = dict(zip(f["checksum_names"].tolist(), f["checksum_values"].tolist()))
    assert sums == want, "regenerated checkpoint differs from the fixture's"
    return cfg, weights, f["lengths"].tolist(), f


def check_against_reference(name, got, f):
    ours = _cos(got, f["emb_fp32"])
    ref_bf16 = _cos(f["emb_bf16"], f["emb_fp32"])
    print(f"{name}: cosine vs fp32 reference: ours min {ours.min():.6f} mean {ours.mean():.6f}; "
          f"reference bf16 min {ref_bf16.min():.6f} mean {ref_bf16.mean():.6f}")
    assert (1 - ours).mean() <= (1 - ref_bf16).mean(), (ours.mean(), ref_bf16.mean())
    assert ours.min() >= min(ref_bf16.min(), 0.9995), (ours.min(), ref_bf16.min())
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    return ours, ref_bf16


def _embed_tp1(cfg, weights, lengths, seed):
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=seed)
    worker = GPUWorker(MESConfig(model_config=cfg), device="cuda:0")
    load_weights(worker.model, weights)
    got = worker.embed(ids, pos, last).numpy()
    assert _C.take_device_error() == 0
    del worker
    torch.cuda.empty_cache()
    return got


def test_c2_qwen3_0_6b_28_layers_20x1000():
    cfg, weights, lengths, f = load_config("c2")
    assert lengths == [1000] * 20 and cfg.num_hidden_layers == 28
    got = _embed_tp1(cfg, weights, lengths, int(f["batch_seed"]))
    check_against_reference("c2", got, f)


def test_c4_slice_qwen3_8b_shapes_with_a_4096_token_sequence():
    cfg, weights, lengths, f = load_config("c4_slice")
    assert max(lengths) == 4096 and cfg.hidden_size == 4096
    got = _embed_tp1(cfg, weights, lengths, int(f["batch_seed"]))
    ours, ref = check_against_reference("c4_slice", got, f)
    assert ours.min() >= 0.9995


def test_c5_qwen2_1_5b_tp1():
    cfg, weights, lengths, f = load_config("c5")
    assert len(lengths) == 64 and cfg.num_hidden_layers == 28
    got = _embed_tp1(cfg, weights, lengths, int(f["batch_seed"]))
    check_against_reference("c5 (tp1)", got, f)


# ------------------------------------------------------------- c5 at TP2 over NCCL
def get_from_ranks(q, procs, timeout: float):
    """The first result a rank puts on ``q``; fails as soon as a rank has exited with an
    error instead of waiting for the whole timeout."""
    import queue
    import time
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        try:
            return q.get(timeout=5)
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead:
                for p in procs:
                    p.join(timeout=30)
                    if p.is_alive():
                        p.kill()
                pytest.fail(f"a rank exited with {dead}")
    for p in procs:
        p.kill()
    pytest.fail("no result from the ranks")


def _tp2_rank(rank, port, q):
    import datetime
    import sys
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from mes_b200.core.gpu_worker import tp_nccl_environment
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    tp_nccl_environment(2)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    worker = None
    try:
        cfg, weights, lengths, f = load_config("c5")
        ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=int(f["batch_seed"]))
        worker = GPUWorker(MESConfig(model_config=cfg), device=dev)
        load_weights(worker.model, weights)     # each rank keeps one of the 2 KV heads
        assert worker.model.model.layers[0].self_attn.num_kv_heads == 1
        got = []
        for graphs in (False, True):                # eager, then a CUDA-graph replay
            worker.use_cuda_graphs = graphs
            got.append(worker.embed(ids, pos, last).numpy())
        assert _C.take_device_error() == 0
        if rank == 0:
            q.put(got)
    finally:
        if worker is not None:
            worker.release_graphs()
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_c5_qwen2_1_5b_tp2_one_kv_head_per_gpu():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp2_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = get_from_ranks(q, procs, timeout=900)
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    # The graph replays the eager forward's kernels; a sum of two ranks' partials is the same
    # whatever algorithm NCCL picks, so the two agree bit for bit.
    assert np.array_equal(got[0], got[1])
    f = np.load(os.path.join(HERE, "golden", "ref_awq_c5.npz"))
    check_against_reference("c5 (tp2)", got[1], f)
