"""patch_aoh_model on small random HF models (head_dim 128), through the CUDA path.

* All heads retrieval: the patched model must give the unpatched model's
  logits (plain causal attention) over chunked prefill and decode.
* Mixed labels (Llama and Qwen3, whose QK-norm the patched forward applies):
  every layer's attention output must match the oracle's head-mixed attention
  on the same post-RoPE q/k/v (bf16 tolerance 2e-2).
"""
import numpy as np
import pytest
import torch

from oracle import aoh_oracle as orc

pytestmark = pytest.mark.gpu

CHUNKS = [96, 160, 1, 1, 1]


def _tiny(kind: str):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    kw = dict(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=128, num_hidden_layers=2,
              intermediate_size=512, vocab_size=128, max_position_embeddings=1024)
    torch.manual_seed(7)
    if kind == "llama":
        m = LlamaForCausalLM(LlamaConfig(**kw))
    else:
        m = Qwen3ForCausalLM(Qwen3Config(**kw))
    return m.to("cuda", torch.bfloat16).eval()


def test_all_retrieval_matches_unpatched_model(cuda_device):
    from transformers import DynamicCache

    from aoh_b200.hf import patch_aoh_model

    model = _tiny("llama")
    ids = torch.randint(0, 128, (1, sum(CHUNKS)), generator=torch.Generator().manual_seed(3)).cuda()
    ref, got = [], []
    with torch.no_grad():
        dc = DynamicCache()
        s = 0
        for c in CHUNKS:
            ref.append(model(input_ids=ids[:, s:s + c], past_key_values=dc, use_cache=True).logits.float())
            s += c
        make_cache, n_ret, n_str = patch_aoh_model(model, np.ones((2, 2)), 16, 48)
        assert n_ret == [2, 2] and n_str == [0, 0]
        cache = make_cache(max_context=512)
        s = 0
        for c in CHUNKS:
            got.append(model(input_ids=ids[:, s:s + c], past_key_values=cache, use_cache=True).logits.float())
            s += c
    assert cache.get_seq_length() == sum(CHUNKS)
    assert cache.paged.device_status() == 0
    for r, g in zip(ref, got):
        err = (r - g).abs().max().item()
        assert err <= 0.05 * r.abs().max().item(), err
        cos = torch.nn.functional.cosine_similarity(r.flatten(), g.flatten(), dim=0).item()
        assert cos > 0.999, cos


@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_mixed_labels_match_oracle(cuda_device, kind, monkeypatch):
    import aoh_b200.hf as hf

    model = _tiny(kind)
    labels = np.array([[1, 0], [0, 1]], dtype=np.float64)
    sink, recent = 16, 48
    oc = orc.OracleKVCache(2, labels, sink, recent, "bf16")
    errs = []
    real = hf.aoh_attention

    def checked(cache, layer, q, k, v, **kw):
        out = real(cache, layer, q, k, v, **kw)
        want = orc.layer_attention(oc, layer, *(x.float().cpu().numpy() for x in (q, k, v)))
        errs.append(float(np.abs(out.float().cpu().numpy() - want).max()))
        return out

    monkeypatch.setattr(hf, "aoh_attention", checked)
    make_cache, _, _ = hf.patch_aoh_model(model, labels, sink, recent)
    cache = make_cache(max_context=512)
    ids = torch.randint(0, 128, (1, sum(CHUNKS)), generator=torch.Generator().manual_seed(4)).cuda()
    with torch.no_grad():
        s = 0
        for c in CHUNKS:
            model(input_ids=ids[:, s:s + c], past_key_values=cache, use_cache=True)
            s += c
    assert len(errs) == 2 * len(CHUNKS)
    assert max(errs) <= 2e-2, errs
    assert cache.paged.device_status() == 0


@pytest.mark.parametrize("norm", [False, True])
def test_rope_qk_matches_the_model_functions(cuda_device, norm):
    """aoh_rope_qk against Qwen3's RMSNorm and apply_rotary_pos_emb run as
    torch ops on the same bf16 inputs: RoPE alone bit for bit; with the norm,
    every value within one bf16 ulp (the mean square is summed in another
    order), nearly all of them equal."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

    from aoh_b200 import rope_qk
    B, C, Hq, G, D = 2, 37, 8, 2, 128
    g = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn((B, C, Hq, D), generator=g, device="cuda").to(torch.bfloat16)
    k = (torch.randn((B, C, G, D), generator=g, device="cuda") * 3).to(torch.bfloat16)
    pos = torch.arange(1000, 1000 + C, device="cuda").float()
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], dim=-1)
    cos = emb.cos()[None].expand(B, C, D).to(torch.bfloat16).contiguous()
    sin = emb.sin()[None].expand(B, C, D).to(torch.bfloat16).contiguous()
    qn = kn = None
    qt, kt = q.transpose(1, 2), k.transpose(1, 2)
    if norm:
        qn, kn = Qwen3RMSNorm(D, eps=1e-6).cuda().to(torch.bfloat16), Qwen3RMSNorm(D, eps=1e-6).cuda().to(torch.bfloat16)
        with torch.no_grad():
            qn.weight.copy_((1 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(torch.bfloat16))
            kn.weight.copy_((1 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(torch.bfloat16))
            qt, kt = qn(qt), kn(kt)
    want_q, want_k = apply_rotary_pos_emb(qt, kt, cos, sin)
    want_q, want_k = want_q.transpose(1, 2), want_k.transpose(1, 2)
    got_q, got_k = rope_qk(q, k, cos, sin, None if qn is None else qn.weight, None if kn is None else kn.weight, 1e-6)
    for got, want in ((got_q, want_q), (got_k, want_k)):
        if not norm:
            assert torch.equal(got, want)
        else:
            w = want.float()
            ulp = torch.where(w == 0, torch.full_like(w, 2.0 ** -133), w.abs() * 2.0 ** -7)
            assert bool(((got.float() - w).abs() <= ulp).all())
            assert (got == want).float().mean().item() > 0.99


@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_decode_graph_matches_eager_steps(cuda_device, kind):
    """ModelDecodeGraph (the whole decode step captured once, the attention on
    the device-resident length) against the same patched model stepped eagerly
    from the same cache contents, token by token: the appended K/V rows (post
    RoPE) are bit-identical -- same positions, same kernels -- and the logits
    agree up to the GEMMs' bf16 rounding (a captured cuBLAS call may use
    another algorithm), at the tolerance of the unpatched-model test above."""
    from aoh_b200.hf import ModelDecodeGraph, patch_aoh_model

    model = _tiny(kind)
    labels = np.array([[1, 0], [0, 1]], dtype=np.float64)
    make_cache, _, _ = patch_aoh_model(model, labels, 16, 48)
    ids = torch.randint(0, 128, (1, 300), generator=torch.Generator().manual_seed(5)).cuda()
    caches = [make_cache(max_context=512) for _ in range(2)]
    want, got = [], []
    with torch.no_grad():
        for c in caches:  # the same prompt in both caches (two chunks, past the window)
            model(input_ids=ids[:, :160], past_key_values=c, use_cache=True)
            model(input_ids=ids[:, 160:290], past_key_values=c, use_cache=True)
        g = ModelDecodeGraph(model, caches[1], max_steps=16)
        for t in range(290, 300):
            want.append(model(input_ids=ids[:, t:t + 1], past_key_values=caches[0], use_cache=True).logits.float())
            got.append(g.step(ids[:, t]).float().clone())
    torch.cuda.synchronize()
    assert caches[0].get_seq_length() == caches[1].get_seq_length() == 300
    for c in caches:
        assert c.paged.device_status() == 0
    for layer in range(2):
        for kv in range(2):
            pos = [290, 295, 299] if labels[layer, kv] >= 0.5 else [295, 299]  # streaming: rows still held
            ka, va = caches[0].paged.read_rows(layer, 0, kv, pos)
            kb, vb = caches[1].paged.read_rows(layer, 0, kv, pos)
            assert torch.equal(ka, kb) and torch.equal(va, vb), (layer, kv)
    for t, (w, gl) in enumerate(zip(want, got)):
        err = (w - gl).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(w.flatten(), gl.flatten(), dim=0).item()
        print(f"step {t}: max abs err {err:.4f} (max |logit| {w.abs().max().item():.3f}), cosine {cos:.6f}")
        assert err <= 0.05 * w.abs().max().item() and cos > 0.999, (t, err, cos)
