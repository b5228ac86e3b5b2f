"""End-to-end parity: the mes_b200 model (CUDA kernels through the C ABI) against the
fp32 dequantised CPU oracle on the same seeded AWQ weights and packed batches.
Criterion: cosine similarity >= 0.9995 per embedding row."""
import numpy as np
import pytest
import torch

from mes_b200 import _C, synthetic
from mes_b200.core.gpu_worker import GPUWorker
from mes_b200.schemas.config import MESConfig
from mes_b200.ultils.loader import load_weights
from oracle import model as omodel

pytestmark = pytest.mark.gpu
COS_MIN = 0.9995


def _run(cfg, lengths, seed=0, norm_noise=0.1):
    weights = synthetic.awq_weights(cfg, seed=seed, device="cpu", norm_noise=norm_noise)
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=seed + 1)
    worker = GPUWorker(MESConfig(model_config=cfg), device="cuda:0")
    load_weights(worker.model, weights)
    got = worker.embed(ids, pos, last).numpy()
    assert _C.take_device_error() == 0
    ref = omodel.embed(cfg, omodel.awq_dense_weights(weights), torch.from_numpy(ids),
                       torch.from_numpy(pos), torch.from_numpy(last),
                       qk_norm=not synthetic.is_qwen2(cfg)).numpy()
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    return cos, got


@pytest.mark.parametrize("lengths", [[128, 128, 128, 128], [1, 17, 200, 333, 64]])
def test_qwen3_0_6b_two_layers(lengths):
    cos, _ = _run(synthetic.qwen3_0_6b(num_hidden_layers=2), lengths)
    assert cos.min() >= COS_MIN, cos


def test_qwen2_1_5b_two_layers():
    cos, _ = _run(synthetic.qwen2_1_5b(num_hidden_layers=2), [16, 100, 511, 7])
    assert cos.min() >= COS_MIN, cos


def test_qwen3_0_6b_full_depth_short_batch():
    cos, got = _run(synthetic.qwen3_0_6b(), [64, 130, 20])
    assert cos.min() >= COS_MIN, cos
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
