"""Hybrid Kernel-DeltaNet LM (20:2 Kernel-DeltaNet : softmax-anchor stack) against the float64 oracle.

CPU: the default model layout (22 blocks, anchors at [10, 21], d_model 2048, 32 x 64 heads,
SwiGLU 8192, vocab 32000), built on the meta device; the oracle LM's own decode identity.
GPU (a tiny model with two anchors; weights re-drawn at a scale where every mixer matters):
  * fp32: ragged prefill logits of every prompt, and the logits of teacher-forced decode
    steps, against the oracle's full-sequence logits (max error <= 1e-4 of the largest logit);
    greedy generation gives the oracle's greedy tokens;
  * bf16 weights and activations (tensor-core prefill): logits within 3e-2;
  * ``forward`` on a uniform batch equals the per-sequence prefill logits.
"""

import numpy as np
import pytest
import torch

import oracle
from oracle import hybrid_lm as olm

TINY = dict(vocab_size=263, d_model=128, num_layers=4, num_heads=2, d_ff=256, anchor_layers=[1, 3])


def test_default_layout_meta():
    from kdn_b200.models import KernelDeltaNetLM

    with torch.device("meta"):
        m = KernelDeltaNetLM()
    kinds = ["anchor" if b.anchor else "kdn" for b in m.layers]
    assert len(kinds) == 22 and [i for i, k in enumerate(kinds) if k == "anchor"] == [10, 21]
    assert m.layers[0].mixer.w_qkvb.weight.shape == (3 * 2048 + 32, 2048)
    assert m.layers[0].ffn.w_gate_up.weight.shape == (2 * 8192, 2048)
    assert m.lm_head.weight is m.embed.weight and m.embed.weight.shape == (32000, 2048)


def _params(model):
    """The model's weights as the oracle's float64 dict."""
    f = lambda t: t.detach().double().cpu().numpy()
    layers = []
    for b in model.layers:
        p = {"anchor": b.anchor, "norm1": f(b.norm1.weight), "norm2": f(b.norm2.weight),
             "w_gate_up": f(b.ffn.w_gate_up.weight), "w_down": f(b.ffn.w_down.weight), "w_out": f(b.mixer.w_out.weight)}
        if b.anchor:
            p["w_qkv"] = f(b.mixer.w_qkv.weight)
        else:
            p["w_qkvb"] = f(b.mixer.w_qkvb.weight)
            p["logit_decay"] = f(b.mixer.logit_decay)
        layers.append(p)
    return {"embed": f(model.embed.weight), "final_norm": f(model.final_norm.weight),
            "lm_head": f(model.lm_head.weight), "layers": layers}


def test_oracle_lm_prefix_consistency():
    """The oracle's logits at position t do not depend on later tokens (causality of every mixer)."""
    rng = np.random.default_rng(3)
    d, H, V, f = 128, 2, 50, 64
    layers = []
    for anchor in (False, True):
        p = {"anchor": anchor, "norm1": 1 + 0.1 * rng.standard_normal(d), "norm2": 1 + 0.1 * rng.standard_normal(d),
             "w_gate_up": rng.standard_normal((2 * f, d)) / np.sqrt(d), "w_down": rng.standard_normal((d, f)) / 8,
             "w_out": rng.standard_normal((d, d)) / np.sqrt(d)}
        if anchor:
            p["w_qkv"] = rng.standard_normal((3 * d, d)) / np.sqrt(d)
        else:
            p["w_qkvb"] = rng.standard_normal((3 * d + H, d)) / np.sqrt(d)
            p["logit_decay"] = rng.uniform(1, 4, H)
        layers.append(p)
    params = {"embed": rng.standard_normal((V, d)), "final_norm": np.ones(d), "lm_head": rng.standard_normal((V, d)),
              "layers": layers}
    c = oracle.make_projection_constants()
    ids = rng.integers(0, V, 90)
    full = olm.lm_logits(params, ids, H, c, 32)
    part = olm.lm_logits(params, ids[:70], H, c, 32)
    assert np.abs(full[:70] - part).max() <= 1e-10 * np.abs(full).max()


def _tiny(dtype, mode, seed=0):
    from kdn_b200.models import KernelDeltaNetLM

    torch.backends.cuda.matmul.allow_tf32 = False  # fp32 GEMMs in fp32 (the oracle is float64)

    torch.manual_seed(seed)
    m = KernelDeltaNetLM(**TINY, mode=mode)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("logit_decay"):
                p.copy_(torch.rand(p.shape, generator=g) * 3 + 1)
            elif "norm" in name:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            elif p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5)
    return m.to("cuda", dtype)


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


@pytest.mark.gpu
def test_prefill_and_decode_match_oracle_fp32():
    m = _tiny(torch.float32, "fp32")
    params = _params(m)
    c = oracle.make_projection_constants()
    rng = np.random.default_rng(7)
    lens = [70, 1, 133]
    prompts = [rng.integers(0, TINY["vocab_size"], n) for n in lens]
    forced = rng.integers(0, TINY["vocab_size"], (len(lens), 4))
    cache = m.new_cache(len(lens), max(lens) + 8)
    cu = np.concatenate([[0], np.cumsum(lens)])
    logits = m.prefill(torch.from_numpy(np.concatenate(prompts)), cu.tolist(), cache).cpu().numpy()
    errs = []
    for i, p in enumerate(prompts):
        errs.append(_rel(logits[i], olm.lm_logits(params, p, TINY["num_heads"], c)[-1]))
    for j in range(forced.shape[1]):
        step = m.decode_step(torch.from_numpy(forced[:, j]).cuda(), cache).cpu().numpy()
        for i, p in enumerate(prompts):
            ref = olm.lm_logits(params, np.concatenate([p, forced[i, :j + 1]]), TINY["num_heads"], c)[-1]
            errs.append(_rel(step[i], ref))
    assert max(errs) <= 1e-4, errs
    assert cache.lengths == [n + forced.shape[1] for n in lens]


@pytest.mark.gpu
def test_greedy_generation_matches_oracle_fp32():
    m = _tiny(torch.float32, "fp32", seed=4)
    params = _params(m)
    c = oracle.make_projection_constants()
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, TINY["vocab_size"], n) for n in (37, 64)]
    out = m.generate([torch.from_numpy(p) for p in prompts], max_new_tokens=5, temperature=0.0)
    for p, o in zip(prompts, out):
        ref = olm.greedy(params, p, 5, TINY["num_heads"], c)
        assert o[len(p):].tolist() == ref
        assert o[:len(p)].tolist() == p.tolist()


@pytest.mark.gpu
def test_bf16_model_close_to_oracle():
    m = _tiny(torch.bfloat16, "bf16", seed=2)
    params = _params(m)  # the oracle runs on the bf16 weights (exactly representable in float64)
    c = oracle.make_projection_constants()
    rng = np.random.default_rng(5)
    lens = [200, 65]
    prompts = [rng.integers(0, TINY["vocab_size"], n) for n in lens]
    cache = m.new_cache(len(lens), max(lens) + 2)
    logits = m.prefill(torch.from_numpy(np.concatenate(prompts)), [0, lens[0], sum(lens)], cache).float().cpu().numpy()
    nxt = rng.integers(0, TINY["vocab_size"], len(lens))
    step = m.decode_step(torch.from_numpy(nxt).cuda(), cache).float().cpu().numpy()
    for i, p in enumerate(prompts):
        full = olm.lm_logits(params, np.concatenate([p, [nxt[i]]]), TINY["num_heads"], c)
        assert _rel(logits[i], full[-2]) <= 3e-2
        assert _rel(step[i], full[-1]) <= 3e-2


@pytest.mark.gpu
def test_forward_uniform_batch_matches_prefill():
    m = _tiny(torch.float32, "fp32", seed=9)
    ids = torch.randint(0, TINY["vocab_size"], (3, 50), generator=torch.Generator().manual_seed(1))
    logits, loss = m(ids, targets=ids)
    last, _ = m.prefill_and_init_states(ids)
    torch.cuda.synchronize()
    assert logits.shape == (3, 50, TINY["vocab_size"]) and torch.isfinite(loss)
    assert float((logits[:, -1] - last[:, 0]).abs().max()) <= 1e-5 * float(last.abs().max())


@pytest.mark.gpu
def test_decode_graph_matches_eager():
    """The captured decode step gives the eager step's logits (teacher-forced) and greedy tokens."""
    m = _tiny(torch.float32, "fp32", seed=6)
    rng = np.random.default_rng(2)
    lens = [40, 90]
    ids = torch.from_numpy(np.concatenate([rng.integers(0, TINY["vocab_size"], n) for n in lens]))
    forced = torch.from_numpy(rng.integers(0, TINY["vocab_size"], (6, 2))).cuda()
    eager, graphed = m.new_cache(2, 100), m.new_cache(2, 100)
    m.prefill(ids, [0, 40, 130], eager)
    m.prefill(ids, [0, 40, 130], graphed)
    g = m.capture_decode(graphed, greedy=False)
    for j in range(6):
        a = m.decode_step(forced[j], eager)
        b = g.step(forced[j])
        assert float((a - b).abs().max()) <= 1e-5 * float(a.abs().max())
    assert eager.lengths == graphed.lengths == [46, 96]
    out_eager = m.generate([ids[:40], ids[40:]], max_new_tokens=6, temperature=0.0, use_graph=False)
    out_graph = m.generate([ids[:40], ids[40:]], max_new_tokens=6, temperature=0.0, use_graph=True)
    assert all(torch.equal(a, b) for a, b in zip(out_eager, out_graph))
