"""Write the golden fixtures of tests/golden/ by running the reference itself on CPU.

Run where a checkout of the reference exists (its directory is given by ``--reference``
or the environment variable ``MES_REFERENCE_DIR``):

    python tests/golden/make_golden.py --reference <reference checkout> [--only NAME ...]

The reference's own Python model code (woodx9/minimal-embedding-server) runs on CPU with
four harness-side adaptations and no change to its sources:
  * a stub module ``sgl_kernel.flash_attn`` whose ``flash_attn_varlen_func`` runs causal
    SDPA per sequence (query head h reads KV head h // (Hq / Hkv)), so the reference's own
    ``FlashAttention.forward`` (cu_seqlens derivation included) stays in the loop;
  * a single-process ``gloo`` process group (its layers call ``dist.get_rank()``);
  * ``config.rope_scaling = None`` (``get_rope`` is lru_cached on it);
  * ``TORCHDYNAMO_DISABLE=1`` (``@torch.compile`` cannot build on this CPU image);
  * ``get_rope.cache_clear()`` before each model build (one process builds several).
For fp32 the reference's ``RMSNorm`` aliases its input (``layers/layernorm.py:23-25,37-39``)
and corrupts the residual; the "fixed" runs pass a copy into it, the "as_is" runs record
the defect.  Weights come from ``mes_b200.synthetic.dense_weights`` (seeded, checkpoint
names) and are loaded through the reference's own ``ultils/loader.load_model``.

Fixtures (all small): ``ref_ops.npz`` (per-op outputs), ``ref_qwen3_c1.npz`` (the 0.6B
architecture, 28 layers, 4 x 128 tokens, fp32), ``ref_qwen2_small.npz`` (Qwen2-1.5B
shapes, 2 layers, ragged batch), ``awq_pack_vllm.npz`` (vLLM 0.22.0 ``awq_pack``).

Benchmark-configuration fixtures (``ref_awq_<config>.npz``): the seeded AWQ checkpoint of
the configuration (codes and zero-points uniform in [0, 15], fp16 scales uniform in
[0.002, 0.02], ``mes_b200.synthetic.awq_weights`` on the CPU generator, so any machine
regenerates it bit for bit; checksums of its tensors are stored to prove that) is
dequantised exactly to fp32 and loaded as the dense weights of the reference's model.
Stored are the reference's last-token L2-normalised embeddings in fp32 (the parity
target, the "fp32 dequantised reference") and in bf16 (the reference's deployment dtype,
whose own distance from fp32 is the yardstick for ours), plus the oracle's fp32
restatement on the same inputs.
  * ``c2``: Qwen3-Embedding-0.6B, 28 layers, 20 x 1000 tokens;
  * ``c4_slice``: Qwen3-Embedding-8B shapes, 2 layers, a 4096-token sequence plus
    log-uniform [64, 4096] lengths (8192 tokens);
  * ``c5``: Qwen2-1.5B, 28 layers, 64 sequences of uniform [16, 512] tokens.
"""
from __future__ import annotations

import os
import sys
import tempfile
import types

os.environ["TORCHDYNAMO_DISABLE"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.nn.functional as F  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REFERENCE = None   # the reference checkout, from --reference / MES_REFERENCE_DIR


def _stub_flash_attn():
    def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                               max_seqlen_k, causal=True):
        rep = q.shape[1] // k.shape[1]
        outs = []
        cu = cu_seqlens_q.tolist()
        for s, e in zip(cu[:-1], cu[1:]):
            qq = q[s:e].transpose(0, 1)
            kk = k[s:e].repeat_interleave(rep, 1).transpose(0, 1)
            vv = v[s:e].repeat_interleave(rep, 1).transpose(0, 1)
            outs.append(F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal).transpose(0, 1))
        return torch.cat(outs, 0)
    pkg = types.ModuleType("sgl_kernel")
    mod = types.ModuleType("sgl_kernel.flash_attn")
    mod.flash_attn_varlen_func = flash_attn_varlen_func
    pkg.flash_attn = mod
    sys.modules["sgl_kernel"] = pkg
    sys.modules["sgl_kernel.flash_attn"] = mod


def _setup_reference():
    if not REFERENCE or not os.path.isdir(REFERENCE):
        raise SystemExit("give the reference checkout with --reference or MES_REFERENCE_DIR")
    _stub_flash_attn()
    sys.path.insert(0, REFERENCE)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=0, world_size=1)


_ORIGINAL = {}


def _fix_rmsnorm_alias():
    """Out-of-place RMSNorm for fp32 runs (the arithmetic of layernorm.py:18-41)."""
    from layers.layernorm import RMSNorm
    if not _ORIGINAL:
        _ORIGINAL["rms"], _ORIGINAL["add"] = RMSNorm.rms_forward, RMSNorm.add_rms_forward

    def rms_forward(self, x):
        return _ORIGINAL["rms"](self, x.clone())

    def add_rms_forward(self, x, residual):
        orig = x.dtype
        s = x.to(torch.float32) + residual.to(torch.float32)
        new_res = s.to(orig).clone()
        var = s.pow(2).mean(dim=-1, keepdim=True)
        return (s * torch.rsqrt(var + self.eps)).to(orig) * self.weight, new_res

    RMSNorm.rms_forward = rms_forward
    RMSNorm.add_rms_forward = add_rms_forward


def _restore_rmsnorm():
    from layers.layernorm import RMSNorm
    if _ORIGINAL:
        RMSNorm.rms_forward, RMSNorm.add_rms_forward = _ORIGINAL["rms"], _ORIGINAL["add"]


def _hf_config(cfg):
    """HF config object for the reference's constructors."""
    from transformers import Qwen2Config, Qwen3Config
    cls = Qwen2Config if cfg.architectures[0] == "Qwen2ForCausalLM" else Qwen3Config
    c = cls(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
            num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
            num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
            intermediate_size=cfg.intermediate_size, rms_norm_eps=cfg.rms_norm_eps,
            max_position_embeddings=cfg.max_position_embeddings, hidden_act="silu")
    c.rope_scaling = None
    c.architectures = list(cfg.architectures)
    return c


def _reference_model(cfg, weights, dtype):
    import models  # noqa: F401  (registers the architectures)
    from models.registry import get_model_class
    from schemas.config import MESConfig
    from ultils.loader import load_model
    from safetensors.torch import save_file
    from layers.rotary_embedding import get_rope
    # get_rope is lru_cached, so every model of this process would share one RoPE module,
    # and `.to(bfloat16)` of one model would round the cos/sin cache of the next: build a
    # fresh one per model.
    get_rope.cache_clear()
    hf = _hf_config(cfg)
    model = get_model_class(hf)(MESConfig(attn_backend="flash_attn", model_config=hf))
    with tempfile.TemporaryDirectory() as d:
        save_file({k: v.contiguous() for k, v in weights.items()}, os.path.join(d, "model.safetensors"))
        load_model(model, d)
    return model.to(dtype).eval()


def _embed(model, ids, pos, last, dtype):
    with torch.no_grad():
        h = model(torch.from_numpy(ids), torch.from_numpy(pos))
    return F.normalize(h[torch.from_numpy(last)].float(), p=2, dim=1).numpy(), h.float().numpy()


def model_fixture(name, cfg, lengths, with_bf16=True):
    from mes_b200 import synthetic
    weights = synthetic.dense_weights(cfg, seed=0)
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=1)
    out = dict(ids=ids, positions=pos, last=last, weight_seed=0)
    _fix_rmsnorm_alias()
    m = _reference_model(cfg, weights, torch.float32)
    out["emb_fp32"], hidden = _embed(m, ids, pos, last, torch.float32)
    out["hidden_fp32_rows"] = hidden[last]
    _restore_rmsnorm()
    m = _reference_model(cfg, weights, torch.float32)
    out["emb_fp32_as_is"], _ = _embed(m, ids, pos, last, torch.float32)
    if with_bf16:
        m = _reference_model(cfg, weights, torch.bfloat16)
        out["emb_bf16"], _ = _embed(m, ids, pos, last, torch.bfloat16)
    np.savez_compressed(os.path.join(HERE, name), **out)
    print(name, {k: v.shape for k, v in out.items() if hasattr(v, "shape")})


@torch.no_grad()
def ops_fixture():
    """Per-op outputs of the reference's layer code on seeded bf16 and fp32 inputs."""
    from layers.activation import SiluAndMul
    from layers.attention.flashattention import FlashAttention
    from layers.layernorm import RMSNorm
    from layers.rotary_embedding import RotaryEmbedding
    g = torch.Generator().manual_seed(11)
    out = {}
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float32, "fp32")):
        x = torch.randn(8, 1024, generator=g).to(dt)
        r = torch.randn(8, 1024, generator=g).to(dt)
        norm = RMSNorm(1024, eps=1e-6)
        norm.weight.data = (1 + 0.1 * torch.randn(1024, generator=g))
        norm = norm.to(dt)
        out[f"rms_x_{tag}"], out[f"rms_r_{tag}"] = x.float().numpy(), r.float().numpy()
        out[f"rms_w_{tag}"] = norm.weight.detach().float().numpy()
        out[f"rms_y_{tag}"] = norm(x.clone()).detach().float().numpy()
        y, res = norm(x.clone(), r.clone())
        out[f"addrms_y_{tag}"], out[f"addrms_res_{tag}"] = y.detach().float().numpy(), res.float().numpy()
        gu = (torch.randn(16, 2 * 256, generator=g) * 3).to(dt)
        out[f"silu_x_{tag}"] = gu.float().numpy()
        out[f"silu_y_{tag}"] = SiluAndMul()(gu).float().numpy()
    # RoPE on a ragged batch (theta 1e6, D = 128), fp32 and bf16-cast cache
    pos = torch.cat([torch.arange(20), torch.arange(33), torch.arange(3) + 1000])
    q = torch.randn(len(pos), 4 * 128, generator=g)
    k = torch.randn(len(pos), 2 * 128, generator=g)
    rope = RotaryEmbedding(128, 128, 4096, 1e6)
    rq, rk = rope(pos, q.clone(), k.clone())
    out.update(rope_pos=pos.numpy(), rope_q=q.numpy(), rope_k=k.numpy(), rope_q_out=rq.numpy(),
               rope_k_out=rk.numpy())
    rope_b = RotaryEmbedding(128, 128, 4096, 1e6).to(torch.bfloat16)
    rqb, rkb = rope_b(pos, q.to(torch.bfloat16), k.to(torch.bfloat16))
    out.update(rope_q_out_bf16=rqb.float().numpy(), rope_k_out_bf16=rkb.float().numpy())
    # Attention backend (cu_seqlens from positions + causal GQA), fp32
    attn = FlashAttention(8, 128, 128 ** -0.5, 2)
    aq = torch.randn(len(pos), 8 * 128, generator=g)
    ak = torch.randn(len(pos), 2 * 128, generator=g)
    av = torch.randn(len(pos), 2 * 128, generator=g)
    out.update(attn_q=aq.numpy(), attn_k=ak.numpy(), attn_v=av.numpy(),
               attn_out=attn(aq, ak, av, pos).numpy())
    np.savez_compressed(os.path.join(HERE, "ref_ops.npz"), **out)
    print("ref_ops.npz", len(out), "arrays")


def awq_pack_fixture():
    from vllm.model_executor.layers.quantization.utils.quant_utils import awq_pack
    rng = np.random.default_rng(5)
    K, N = 256, 64
    codes = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    packed = awq_pack(torch.from_numpy(codes.astype(np.int32)), 4, K, N).numpy()
    np.savez_compressed(os.path.join(HERE, "awq_pack_vllm.npz"), codes=codes, packed=packed)
    print("awq_pack_vllm.npz", packed.shape, packed.dtype)


# Benchmark configurations of the AWQ parity fixtures: (architecture, overrides,
# lengths, weight seed, batch seed, norm noise).
def awq_configs():
    from mes_b200 import synthetic
    c4_lengths = [4096] + synthetic.lengths_log_uniform(4096, 64, 4096, seed=3)
    return {
        "c2": (synthetic.qwen3_0_6b, dict(max_position_embeddings=32768), [1000] * 20, 0, 1, 0.1),
        "c4_slice": (synthetic.qwen3_8b, dict(num_hidden_layers=2, max_position_embeddings=32768),
                     c4_lengths, 0, 1, 0.1),
        "c5": (synthetic.qwen2_1_5b, dict(max_position_embeddings=32768),
               synthetic.lengths_uniform(64, 16, 512, seed=1), 0, 1, 0.1),
    }


def weight_checksums(weights: dict) -> dict:
    """Exact integer checksums of every AWQ tensor and the embedding table's bits: a
    regenerated checkpoint matches the fixture's only if every sum matches."""
    out = {}
    for name in sorted(weights):
        t = weights[name]
        if t.dtype in (torch.float16, torch.bfloat16):
            t = t.view(torch.int16)
        out[name] = int(t.to(torch.int64).sum())
    return out


def awq_config_fixture(name):
    from mes_b200 import synthetic
    sys.path.insert(0, REPO)
    from oracle import model as omodel
    arch, over, lengths, wseed, bseed, noise = awq_configs()[name]
    cfg = arch(**over)
    weights = synthetic.awq_weights(cfg, seed=wseed, device="cpu", norm_noise=noise)
    sums = weight_checksums(weights)
    dense = omodel.awq_dense_weights(weights)
    del weights
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=bseed)
    qk = not synthetic.is_qwen2(cfg)
    out = dict(lengths=np.asarray(lengths, dtype=np.int64), weight_seed=wseed, batch_seed=bseed,
               norm_noise=noise, checksum_names=np.asarray(list(sums)),
               checksum_values=np.asarray(list(sums.values()), dtype=np.int64))
    out["emb_oracle_fp32"] = omodel.embed(cfg, dense, torch.from_numpy(ids), torch.from_numpy(pos),
                                          torch.from_numpy(last), qk_norm=qk).numpy()
    _fix_rmsnorm_alias()
    m = _reference_model(cfg, dense, torch.float32)
    out["emb_fp32"], _ = _embed(m, ids, pos, last, torch.float32)
    del m
    _restore_rmsnorm()
    m = _reference_model(cfg, dense, torch.bfloat16)
    out["emb_bf16"], _ = _embed(m, ids, pos, last, torch.bfloat16)
    del m
    path = os.path.join(HERE, f"ref_awq_{name}.npz")
    np.savez_compressed(path, **out)
    cos = lambda a, b: (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    print(path, "reference bf16 vs fp32 cosine min", cos(out["emb_bf16"], out["emb_fp32"]).min(),
          "oracle vs reference fp32 min", cos(out["emb_oracle_fp32"], out["emb_fp32"]).min())


def main():
    import argparse
    global REFERENCE
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MES_REFERENCE_DIR"),
                    help="directory of the reference checkout")
    ap.add_argument("--only", nargs="*", default=None,
                    help="fixtures to write (ops, c1, qwen2_small, awq_pack, c2, c4_slice, c5)")
    args = ap.parse_args()
    REFERENCE = args.reference
    sys.path.insert(0, REPO)
    import __graft_entry__
    __graft_entry__.load_package()
    from mes_b200 import synthetic
    _setup_reference()
    torch.set_num_threads(os.cpu_count() or 1)
    want = set(args.only) if args.only else None

    def on(name):
        return want is None or name in want

    if on("awq_pack"):
        awq_pack_fixture()
    if on("ops"):
        ops_fixture()
    if on("c1"):
        model_fixture("ref_qwen3_c1.npz", synthetic.qwen3_0_6b(max_position_embeddings=32768),
                      [128, 128, 128, 128])
    if on("qwen2_small"):
        model_fixture("ref_qwen2_small.npz",
                      synthetic.qwen2_1_5b(num_hidden_layers=2, max_position_embeddings=32768),
                      [1, 17, 64, 200])
    for name in awq_configs():
        if on(name):
            awq_config_fixture(name)


if __name__ == "__main__":
    main()
