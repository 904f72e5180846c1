"""Host-side pieces of the package drop-in (CPU): the store's on-disk .u8 format and its builders'
bookkeeping, the cache's copy coalescing, and how attach() fits the HF decoder layer it lands in."""

import os

import numpy as np
import pytest
import torch

from wisp import quant
from wisp.cache import ExpertCache
from wisp.store import ExpertStore


def test_store_file_is_the_raw_host_array(tmp_path):
    """_save writes the host array byte for byte under the reference's file name, via a .tmp file and a
    rename; _load / load read it back (wisp/store.py:54-110)."""
    st = ExpertStore(2, 3, 2048, 4, 128, pin=False)
    rng = np.random.default_rng(0)
    st.host.numpy()[:] = rng.integers(0, 256, st.host.shape, dtype=np.uint8)
    path = st.cache_path(str(tmp_path))
    assert os.path.basename(path) == "store_b4_g128_2x3x2048.u8"
    st._save(path, rows=2)
    assert not os.path.exists(path + ".tmp")
    raw = np.fromfile(path, dtype=np.uint8)
    assert raw.size == st.host.numel() and np.array_equal(raw, st.host.numpy().reshape(-1))
    back = ExpertStore.load(path, 2, 3, 2048, 4, 128, pin=False)
    assert torch.equal(back.host, st.host)
    assert back.nbytes == quant.expert_nbytes(2048, 4, 128) and back.key(1, 2) == 5
    short = tmp_path / "short.u8"
    short.write_bytes(b"\0" * 10)
    with pytest.raises(ValueError):
        back._load(str(short))


def test_store_from_pool_and_shape_names():
    n, bits, group, L, E = 2048, 3, 128, 2, 4
    nb = quant.expert_nbytes(n, bits, group)
    pool = torch.arange(L * E * nb, dtype=torch.int64).remainder(251).to(torch.uint8).reshape(L * E, nb)
    st = ExpertStore.from_pool(pool, n, bits, group, L, E, pin=False)
    assert torch.equal(st.host, pool)
    assert (st.L, st.E, st.layers, st.experts, st.nbytes) == (L, E, L, E, nb)
    assert st.total_gib == pytest.approx(pool.numel() / 2**30)
    with pytest.raises(AssertionError):
        ExpertStore.from_pool(pool[:-1], n, bits, group, L, E, pin=False)


def test_copy_runs_coalesce_consecutive_keys_and_slots():
    runs = ExpertCache._runs([(5, 0), (6, 1), (7, 2), (9, 3), (10, 4), (3, 7), (4, 9)])
    assert runs == [(5, 0, 3), (9, 3, 2), (3, 7, 1), (4, 9, 1)]
    assert ExpertCache._runs([]) == []
    # every (key, slot) is covered exactly once
    pairs = [(k, s) for k0, s0, n in runs for k, s in zip(range(k0, k0 + n), range(s0, s0 + n))]
    assert pairs == [(5, 0), (6, 1), (7, 2), (9, 3), (10, 4), (3, 7), (4, 9)]


def test_attach_fits_the_decoder_layer():
    """transformers 5 Qwen3-MoE layers add the MLP output straight to the residual, so the attached
    blocks return a tensor there; a layer that unpacks (hidden, router_logits) gets the tuple."""
    transformers = pytest.importorskip("transformers")
    from wisp.moe import PagedMoEBlock, Runtime, _layer_unpacks_tuple, attach

    cfg = transformers.Qwen3MoeConfig(vocab_size=32, hidden_size=64, intermediate_size=64, moe_intermediate_size=32,
                                      num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                                      num_experts=4, num_experts_per_tok=2, norm_topk_prob=True)
    model = transformers.AutoModelForCausalLM.from_config(cfg)
    rt = Runtime(None)
    attach(model, rt)
    blocks = [layer.mlp for layer in model.model.layers]
    assert all(isinstance(b, PagedMoEBlock) for b in blocks)
    assert blocks[0].next_gate is blocks[1].gate and blocks[1].next_gate is None
    want = _layer_unpacks_tuple(model.model.layers[0])
    assert all(b.return_logits == want for b in blocks)
    assert "next_gate" not in dict(blocks[0].named_modules())  # the next layer's gate is not registered here

    class Old(torch.nn.Module):
        def forward(self, hidden_states):
            hidden_states = self.mlp(hidden_states)
            if isinstance(hidden_states, tuple):
                hidden_states, router_logits = hidden_states
            return hidden_states

    assert _layer_unpacks_tuple(Old())


def test_runtime_reads_wisp_fused(monkeypatch):
    from wisp.moe import Runtime

    monkeypatch.setenv("WISP_FUSED", "2")
    assert Runtime(None).fused == 2
    monkeypatch.setenv("WISP_FUSED", "0")
    assert Runtime(None, fused=1).fused == 1
    assert Runtime(None).stats == dict(layer_calls=0, cpu_experts=0, gpu_experts=0, cpu_time=0.0, admitted=0, prefetched=0)


def test_mxfp4_decode_matches_hf():
    """MXFP4 blocks/scales -> bf16, bit-exact with HF's convert_moe_packed_tensors (the reference test
    tests/test_gptoss.py:10-16), signed zeros included."""
    pytest.importorskip("transformers")
    from transformers.integrations.mxfp4 import convert_moe_packed_tensors

    from wisp.gptoss import expert_w3, mxfp4_to_bf16

    g = torch.Generator().manual_seed(0)
    blocks = torch.randint(0, 256, (2, 6, 4, 16), dtype=torch.uint8, generator=g)
    scales = torch.randint(118, 136, (2, 6, 4), dtype=torch.uint8, generator=g)
    ours = mxfp4_to_bf16(blocks, scales)
    hf = convert_moe_packed_tensors(blocks, scales)  # [E, K, out]
    assert torch.equal(ours.transpose(1, 2).contiguous().view(torch.int16), hf.contiguous().view(torch.int16))
    gu, dn = torch.randn(8, 16), torch.randn(8, 8)
    w3 = expert_w3(gu, dn)
    assert w3.shape == (3, 64) and torch.equal(w3[0], gu.reshape(-1)[:64]) and torch.equal(w3[2], dn.reshape(-1))
