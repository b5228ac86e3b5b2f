"""Tensor-parallel host logic on CPU: two ``gloo`` ranks build the mes_b200 model, load one
AWQ checkpoint through its ``weight_loader``s (column shards on the packed N axis, row
shards on K and K/G), and run the oracle's TP forward on exactly the shards each rank
holds, with the all-reduce after o_proj and down_proj.  The result must equal the TP=1
forward on the full weights.  No GPU is involved (the kernels are not called)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shards_to_dense(model, cfg):
    """This rank's AWQ shards -> oracle-named dense fp32 weights ([out_local, in_local])."""
    from oracle import awq as oawq

    def deq(lin):
        w = oawq.dequant_fp32(lin.qweight.numpy(), lin.qzeros.numpy(),
                              lin.scales.view(torch.float16).numpy())
        return torch.from_numpy(np.ascontiguousarray(w.T))  # [N_local, K_local]

    m = model.model
    W = {"embed_tokens.weight": m.embed_tokens.weight.float(), "norm.weight": m.norm.weight.float()}
    for i, layer in enumerate(m.layers):
        p = f"layers.{i}."
        at, mlp = layer.self_attn, layer.mlp
        W[p + "input_layernorm.weight"] = layer.input_layernorm.weight.float()
        W[p + "post_attention_layernorm.weight"] = layer.post_attention_layernorm.weight.float()
        W[p + "self_attn.q_norm.weight"] = at.q_norm.weight.float()
        W[p + "self_attn.k_norm.weight"] = at.k_norm.weight.float()
        qkv = deq(at.qkv_proj)
        nq, nk = at.q_size, at.kv_size
        for name, part in zip(("q", "k", "v"), qkv.split([nq, nk, nk])):
            W[p + f"self_attn.{name}_proj.weight"] = part
        if at.qkv_proj.bias is not None:
            for name, part in zip(("q", "k", "v"), at.qkv_proj.bias.float().split([nq, nk, nk])):
                W[p + f"self_attn.{name}_proj.bias"] = part
        W[p + "self_attn.o_proj.weight"] = deq(at.o_proj)
        gate, up = deq(mlp.gate_up_proj).chunk(2, 0)
        W[p + "mlp.gate_proj.weight"], W[p + "mlp.up_proj.weight"] = gate, up
        W[p + "mlp.down_proj.weight"] = deq(mlp.down_proj)
    return W


def _worker(rank, world, port, arch, result_q):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from mes_b200 import synthetic
    from mes_b200.models import Qwen2ForCausalLM, Qwen3ForCausalLM
    from mes_b200.schemas.config import MESConfig
    from mes_b200.ultils.loader import load_weights
    from oracle import model as omodel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(2)
    try:
        if arch == "qwen3":
            cfg = synthetic.qwen3_0_6b(num_hidden_layers=2, vocab_size=1000)
            cls = Qwen3ForCausalLM
        else:
            cfg = synthetic.qwen2_1_5b(num_hidden_layers=2, vocab_size=1000)
            cls = Qwen2ForCausalLM
        ckpt = synthetic.quantize_dense_checkpoint(synthetic.dense_weights(cfg, seed=0))
        model = cls(MESConfig(model_config=cfg))
        load_weights(model, ckpt)                       # the product's sharding logic
        ids, pos, last = synthetic.packed_batch([5, 40, 17], cfg.vocab_size, seed=2)
        ids, pos, last = map(torch.from_numpy, (ids, pos, last))
        qk = arch == "qwen3"
        tp = omodel.embed(cfg, _shards_to_dense(model, cfg), ids, pos, last, qk_norm=qk,
                          world=world)
        full = omodel.embed(cfg, omodel.awq_dense_weights(ckpt), ids, pos, last, qk_norm=qk)
        result_q.put((rank, float((tp - full).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("arch,world", [("qwen3", 2), ("qwen2", 2), ("qwen3", 4), ("qwen3", 8)])
def test_tp_shards_reproduce_tp1(arch, world):
    # Qwen3-0.6B at TP 4 / 8: 4 / 2 q heads and 2 / 1 kv heads per rank; down_proj's K
    # shard is 768 / 384 (6 / 3 AWQ groups).
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, arch, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = dict(q.get(timeout=10) for _ in range(world))
    assert max(results.values()) < 1e-5, results


def test_overlap_split_is_a_sequence_start_near_the_middle(monkeypatch):
    import numpy as np
    from mes_b200.models import qwen2
    monkeypatch.setattr(qwen2, "_tp_size", lambda: 2)
    pos = np.concatenate([np.arange(n) for n in (1000, 700, 1300, 1000, 1000)])
    assert qwen2.DecoderModel.overlap_split_host(pos) == 3000     # starts 1000, 1700, 3000, 4000
    NO = qwen2.DecoderModel.NO_SPLIT
    assert qwen2.DecoderModel.overlap_split_host(np.arange(5000)) == NO         # one sequence
    assert qwen2.DecoderModel.overlap_split_host(np.arange(100)) == NO          # below the threshold
    # A micro-batch of 256 tokens or fewer is never cut off (its GEMMs would split K).
    edge = np.concatenate([np.arange(4800), np.arange(200)])
    assert qwen2.DecoderModel.overlap_split_host(edge) == NO
    edge = np.concatenate([np.arange(200), np.arange(2000), np.arange(2800)])
    assert qwen2.DecoderModel.overlap_split_host(edge) == 2200
    # The model's own path (positions as a torch tensor) applies the same rule.
    import torch
    import types
    D = qwen2.DecoderModel
    m = types.SimpleNamespace(tp_size=2, overlap_min_tokens=D.overlap_min_tokens,
                              _nearest_middle=D._nearest_middle)
    assert D._overlap_split(m, torch.from_numpy(pos)) == 3000
    assert D._overlap_split(m, torch.from_numpy(np.concatenate([np.arange(4800), np.arange(200)]))) is None
    monkeypatch.setattr(qwen2, "_tp_size", lambda: 1)
    assert qwen2.DecoderModel.overlap_split_host(pos) == NO                    # tp == 1
    assert qwen2.DecoderModel.overlap_reserved_sms(2) == 16
    assert qwen2.DecoderModel.overlap_reserved_sms(8) == 32


def test_host_split_is_used_as_given(monkeypatch):
    """A boundary the host worked out - including "none" for a 4096+-token single sequence -
    is used without the device read (which a CUDA-graph capture forbids); only an absent
    one is derived from the positions."""
    import numpy as np
    import torch
    from mes_b200.models import qwen2
    monkeypatch.setattr(qwen2, "_tp_size", lambda: 2)
    D = qwen2.DecoderModel
    one_seq = np.arange(8192)
    host = D.overlap_split_host(one_seq)
    assert host == D.NO_SPLIT

    def no_device_read(*args):
        raise AssertionError("device read of the split")
    import types
    model = types.SimpleNamespace(tp_size=2, _overlap_split=no_device_read)
    pos_t = torch.from_numpy(one_seq)
    assert D._resolve_split(model, pos_t, host) is None
    assert D._resolve_split(model, pos_t, 3000) == 3000
    with pytest.raises(AssertionError):
        D._resolve_split(model, pos_t, None)
    model.tp_size = 1                     # e.g. a data-parallel replica in a process group
    assert D._resolve_split(model, pos_t, None) is None
    assert D.overlap_split_host(one_seq, tp_size=1) == D.NO_SPLIT
