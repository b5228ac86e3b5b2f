"""GPU-worker host logic on CPU: token buckets, the padded device layout of a host batch
(dummy sequences after each micro-batch, host rows mapped to device rows), the choice
between bucketed and exact graph layouts, and - through the oracle forward - that the
padding leaves every real sequence's embedding unchanged.  No kernel is called."""
import types

import numpy as np
import pytest
import torch

from mes_b200 import synthetic
from mes_b200.core import gpu_worker as gw
from mes_b200.models import qwen2
from oracle import model as omodel
from oracle import ops


def _worker(tp_size: int) -> gw.GPUWorker:
    stub = types.SimpleNamespace(tp_size=tp_size)
    stub.eval = lambda: stub
    return gw.GPUWorker(None, device="cpu", model=stub)


def test_token_bucket_steps():
    cases = {0: 256, 1: 256, 256: 256, 257: 512, 20000: 20224, 32768: 32768,
             32769: 34816, 131072: 131072, 131073: 139264}
    for n, want in cases.items():
        assert gw.token_bucket(n) == want, n
    for n in (1, 255, 1000, 32767, 40000, 131071, 200000):
        b = gw.token_bucket(n)
        step = 256 if n <= 32768 else 2048 if n <= 131072 else 8192
        assert b >= n and b % step == 0 and b - n < step


@pytest.mark.parametrize("tp,lengths", [
    (1, [5, 40, 17, 100]),
    (1, [256, 512]),                      # a bucket size already: no padding
    (2, [1000, 700, 1300, 1000, 1000]),   # split at the sequence start 3000
    (2, [8192]),                          # one sequence: unsplit at tp = 2
])
def test_layout_pads_each_micro_batch_with_new_sequences(monkeypatch, tp, lengths):
    monkeypatch.setattr(qwen2, "_tp_size", lambda: tp)
    ids, pos, last = synthetic.packed_batch(lengths, 1000, seed=3)
    T = len(ids)
    lay = _worker(tp).layout(pos)
    host_split = qwen2.DecoderModel.overlap_split_host(pos, tp)
    spans = [(0, T)] if host_split == qwen2.DecoderModel.NO_SPLIT else [(0, host_split), (host_split, T)]
    assert [(p[0], p[1]) for p in lay.parts] == spans
    d0 = 0
    for s0, s1, dst, n in lay.parts:
        assert dst == d0 and n == gw.token_bucket(s1 - s0)
        d0 += n
    assert lay.total == d0
    assert lay.split == (qwen2.DecoderModel.NO_SPLIT if len(spans) == 1 else lay.parts[1][2])
    assert lay.padded == any(p[3] != p[1] - p[0] for p in lay.parts)

    pids, ppos = lay.pad(ids, pos)
    assert len(pids) == len(ppos) == lay.total
    rows = lay.rows(np.arange(T))
    assert np.array_equal(pids[rows], ids) and np.array_equal(ppos[rows], pos)
    # Sequence boundaries of the device batch: the host's (mapped), each micro-batch start,
    # and dummy sequences of at most PAD_SEQ tokens filling every micro-batch's tail.
    cu = ops.cu_seqlens_from_positions(torch.from_numpy(ppos)).numpy()
    host_cu = ops.cu_seqlens_from_positions(torch.from_numpy(pos)).numpy()
    assert set(lay.rows(host_cu[:-1]).tolist()) <= set(cu.tolist())
    real = np.zeros(lay.total, dtype=bool)
    real[rows] = True
    for a, b in zip(cu[:-1], cu[1:]):
        if not real[a]:
            assert not real[a:b].any() and b - a <= gw.PAD_SEQ and ppos[a] == 0
    # The device micro-batch boundary is a sequence start.
    if lay.split != qwen2.DecoderModel.NO_SPLIT:
        assert lay.split in cu.tolist()
    # Last-token rows stay last tokens on the device.
    for r in lay.rows(last):
        nxt = r + 1
        assert nxt == lay.total or ppos[nxt] != ppos[r] + 1
    # Index tensors map on their own device, to the same rows.
    got = lay.rows(torch.from_numpy(last).to(torch.int32))
    assert got.dtype == torch.int64 and np.array_equal(got.numpy(), lay.rows(last))


def test_exact_layout_is_unpadded():
    ids, pos, _ = synthetic.packed_batch([5, 40, 17], 1000, seed=3)
    lay = _worker(1).layout(pos, exact=True)
    assert not lay.padded and lay.total == len(ids)
    pids, ppos = lay.pad(ids, pos)
    assert pids is ids and ppos is pos
    assert np.array_equal(lay.rows([0, 61]), [0, 61])


def test_graph_layout_is_bucketed_until_a_shape_repeats():
    w = _worker(1)
    _, pos, _ = synthetic.packed_batch([5, 40, 17, 100], 1000, seed=3)
    for i in range(1, w.exact_after):
        lay = w._graph_layout(pos)
        assert lay.padded and lay.total == 256, i
    lay = w._graph_layout(pos)              # the exact_after-th occurrence
    assert not lay.padded and lay.total == 162
    _, pos256, _ = synthetic.packed_batch([200, 56], 1000, seed=3)
    lay = _worker(1)._graph_layout(pos256)   # needs no padding: exact at once
    assert not lay.padded and lay.total == 256


@pytest.mark.parametrize("tp,lengths", [(1, [5, 40, 17, 100, 1]), (2, [1000, 700, 1300, 1000, 1000])])
def test_padding_leaves_real_embeddings_unchanged(monkeypatch, tp, lengths):
    """The oracle forward over the padded device batch, pooled at the mapped rows, equals the
    forward over the host batch (fp32; only the summation blocking of the larger matrices
    differs)."""
    monkeypatch.setattr(qwen2, "_tp_size", lambda: tp)
    cfg = synthetic.qwen3_0_6b(num_hidden_layers=2, vocab_size=500, hidden_size=128,
                               num_attention_heads=2, num_key_value_heads=1, head_dim=64,
                               intermediate_size=256)
    W = synthetic.dense_weights(cfg, seed=4, std=0.05)
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=5)
    lay = _worker(tp).layout(pos)
    assert lay.padded
    pids, ppos = lay.pad(ids, pos)
    want = omodel.embed(cfg, W, torch.from_numpy(ids), torch.from_numpy(pos), last)
    got = omodel.embed(cfg, W, torch.from_numpy(pids), torch.from_numpy(ppos), lay.rows(last))
    torch.testing.assert_close(got, want, rtol=0, atol=1e-5)


def test_empty_batch_launches_nothing():
    def fail(*a, **k):
        raise AssertionError("the model ran for an empty batch")
    stub = types.SimpleNamespace(tp_size=1, forward_last_rows=fail)
    stub.eval = lambda: stub
    cfg = types.SimpleNamespace(model_config=types.SimpleNamespace(hidden_size=64))
    w = gw.GPUWorker(cfg, device="cpu", model=stub)
    w.model = fail
    empty = np.zeros(0, dtype=np.int64)
    emb = w.embed(empty, empty, [])
    assert emb.shape == (0, 64) and emb.dtype == torch.float32
    assert w.embed_list(empty, empty, []) == []
    hidden = w._inference(empty, empty)
    assert hidden.shape == (0, 64) and hidden.dtype == torch.bfloat16
