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
