"""patch_aoh_model host logic (no GPU): argument errors as in the reference
(eval/efficiency/benchmark_llama31.py:257-265), per-layer head counts, and
layers falling through to their original forward for other caches."""
import numpy as np
import pytest
import torch


def _tiny():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=2, head_dim=128,
                      num_hidden_layers=3, intermediate_size=128, vocab_size=32)
    return LlamaForCausalLM(cfg).eval()


def test_patch_validates_arguments():
    from aoh_b200.hf import patch_aoh_model
    m = _tiny()
    with pytest.raises(ValueError):
        patch_aoh_model(m, np.ones((2, 2)), 128, 256)  # wrong number of layers
    with pytest.raises(ValueError):
        patch_aoh_model(m, np.ones((3, 2)), -1, 256)
    make_cache, n_ret, n_str = patch_aoh_model(m, np.array([[1, 0], [0, 0], [1, 1]]), 128, 256)
    assert n_ret == [1, 0, 2] and n_str == [1, 2, 0]
    with pytest.raises(ValueError):  # "eager" and "flash" are the reference's two protocols
        make_cache("fused")


def test_other_caches_use_the_original_forward():
    from transformers import DynamicCache

    from aoh_b200.hf import patch_aoh_model
    m = _tiny()
    ids = torch.randint(0, 32, (1, 9), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        before = m(input_ids=ids, past_key_values=DynamicCache(), use_cache=True).logits
        patch_aoh_model(m, np.ones((3, 2)), 16, 48)
        after = m(input_ids=ids, past_key_values=DynamicCache(), use_cache=True).logits
    assert torch.equal(before, after)


def test_cache_adapter_hooks():
    import types

    from aoh_b200.hf import AoHModelCache
    stub = types.SimpleNamespace(num_layers=2, kv_seq_len=40)
    c = AoHModelCache(stub)
    assert c.get_seq_length() == 40
    assert c.get_mask_sizes(7, 0) == (47, 0)
    assert c.get_mask_sizes(torch.arange(40, 45), 1) == (45, 0)
    k = torch.zeros(1)
    assert c.update(k, k, 0)[0] is k
    c.kv_seq_len = 41
    assert stub.kv_seq_len == 41
