"""AWQ checkpoint loading from safetensors files (``ultils/loader.py:12-33``) on CPU: the
reference's name routing (``model.`` prefix optional, packed q/k/v and gate/up shards
through the packed parameter's ``weight_loader``) over a snapshot split into several
files gives the same parameters as loading the tensors directly, and a name the model does
not have raises as it does in the reference."""
import os

import pytest
import torch
from safetensors.torch import save_file

from mes_b200 import synthetic
from mes_b200.models import Qwen2ForCausalLM, Qwen3ForCausalLM
from mes_b200.schemas.config import MESConfig
from mes_b200.ultils.loader import load_model, load_weights


def _params(model):
    return {n: p.detach().clone() for n, p in model.named_parameters()}


@pytest.mark.parametrize("arch", ["qwen3", "qwen2"])
def test_load_model_from_safetensors_snapshot(tmp_path, arch):
    if arch == "qwen3":
        cfg, cls = synthetic.qwen3_0_6b(num_hidden_layers=2, vocab_size=1000), Qwen3ForCausalLM
    else:
        cfg, cls = synthetic.qwen2_1_5b(num_hidden_layers=2, vocab_size=1000), Qwen2ForCausalLM
    weights = synthetic.awq_weights(cfg, seed=3)
    # Three shards; half of the names carry the "model." prefix, as exported checkpoints do.
    names = sorted(weights)
    for i in range(3):
        part = {(f"model.{n}" if j % 2 else n): weights[n].contiguous()
                for j, n in enumerate(names) if j % 3 == i}
        save_file(part, os.path.join(tmp_path, f"model-0000{i + 1}-of-00003.safetensors"))

    from_files = cls(MESConfig(model_config=cfg))
    load_model(from_files, str(tmp_path))
    direct = cls(MESConfig(model_config=cfg))
    load_weights(direct, weights)
    a, b = _params(from_files), _params(direct)
    assert a.keys() == b.keys()
    for n in a:
        assert torch.equal(a[n], b[n]), n
    # Every checkpoint tensor reached a parameter: the packed q/k/v and gate/up slices.
    at = from_files.model.layers[1].self_attn
    D, nq = at.head_dim, at.num_heads
    qw = at.qkv_proj.qweight
    assert torch.equal(qw[:, : nq * D // 8], weights["layers.1.self_attn.q_proj.qweight"])
    gu = from_files.model.layers[0].mlp.gate_up_proj.scales
    up = weights["layers.0.mlp.up_proj.scales"]
    assert torch.equal(gu.view(torch.float16)[:, up.shape[1]:], up)


def test_unknown_checkpoint_name_raises(tmp_path):
    cfg = synthetic.qwen3_0_6b(num_hidden_layers=1, vocab_size=1000)
    save_file({"model.layers.0.not_a_parameter": torch.zeros(4)},
              os.path.join(tmp_path, "model.safetensors"))
    with pytest.raises(AttributeError):
        load_model(Qwen3ForCausalLM(MESConfig(model_config=cfg)), str(tmp_path))
