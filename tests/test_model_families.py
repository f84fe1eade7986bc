"""Model families (C18): for each supported HF ``model_type`` a tiny random
HF model is saved with ``save_pretrained``; the framework reads its config and
safetensors, and its fused decoder must give the same logits as the HF
implementation (fp32, CPU).  The way back: ``save_hf`` of the framework's
model loads into HF with the same logits.  The rollout engine's greedy tokens
match the training model's argmax on the same prompts."""

import pytest
import torch

transformers = pytest.importorskip("transformers")

SMALL = dict(vocab_size=160, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, max_position_embeddings=512)


def _configs():
    T = transformers
    return {
        "qwen2": lambda: T.Qwen2Config(**SMALL),
        "qwen3": lambda: T.Qwen3Config(**SMALL, head_dim=16),
        "llama": lambda: T.LlamaConfig(**SMALL, head_dim=16, rope_parameters={
            "rope_type": "llama3", "rope_theta": 500000.0, "factor": 8.0, "low_freq_factor": 1.0,
            "high_freq_factor": 4.0, "original_max_position_embeddings": 64}),
        "mistral": lambda: T.MistralConfig(**SMALL, head_dim=16, sliding_window=None),
        "mixtral": lambda: T.MixtralConfig(**SMALL, num_local_experts=4, num_experts_per_tok=2),
        "qwen2_moe": lambda: T.Qwen2MoeConfig(**SMALL, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32,
                                              shared_expert_intermediate_size=48),
        "qwen3_moe": lambda: T.Qwen3MoeConfig(**SMALL, head_dim=16, num_experts=4, num_experts_per_tok=2,
                                              moe_intermediate_size=32),
        "olmoe": lambda: T.OlmoeConfig(**SMALL, num_experts=4, num_experts_per_tok=2),
        "phi3": lambda: T.Phi3Config(**SMALL, pad_token_id=0),
        "gemma": lambda: T.GemmaConfig(**SMALL, head_dim=16),
    }


FAMILIES = list(_configs())


def _hf_model(name, path):
    cfg = _configs()[name]()
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    m = transformers.AutoModelForCausalLM.from_config(cfg).float().eval()
    with torch.no_grad():   # norms away from 1 and non-zero biases exercise every mapping
        for n, p in m.named_parameters():
            if n.endswith("norm.weight") or "layernorm" in n:
                p.copy_(torch.rand_like(p) * 0.5 + (0.75 if name != "gemma" else -0.25))
            elif n.endswith("bias"):
                p.copy_(torch.randn_like(p) * 0.1)
            elif p.dim() >= 2:
                p.copy_(torch.randn_like(p) * 0.08)
    m.save_pretrained(path)
    return m


def _ours(path):
    import json
    from psrl_b200.models import build_model
    from psrl_b200.models.config import ModelArgs
    from psrl_b200.models.hf_io import load_hf_into
    with open(f"{path}/config.json") as fh:
        a = ModelArgs.from_hf_config(json.load(fh))
    m = build_model(a, "cpu", torch.float32)
    load_hf_into(m, str(path))
    return m.eval()


def _our_logits(m, seqs):
    from psrl_b200.models import packed_positions
    ids = torch.cat(seqs)
    pos, cu, mx = packed_positions([len(s) for s in seqs], "cpu")
    with torch.no_grad():
        return m.logits(ids, pos, cu, mx).float()


def _hf_logits(m, seqs):
    with torch.no_grad():
        return torch.cat([m(input_ids=s[None]).logits[0].float() for s in seqs])


@pytest.mark.parametrize("name", FAMILIES)
def test_family_logits_match_hf(name, tmp_path):
    hf = _hf_model(name, tmp_path / "hf")
    ours = _ours(tmp_path / "hf")
    assert ours.args.arch == name
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(1, 160, (n,), generator=g) for n in (23, 9)]
    ref, got = _hf_logits(hf, seqs), _our_logits(ours, seqs)
    torch.testing.assert_close(got, ref, rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("name", FAMILIES)
def test_family_save_loads_into_hf(name, tmp_path):
    from psrl_b200.models.hf_io import save_hf
    _hf_model(name, tmp_path / "hf")
    ours = _ours(tmp_path / "hf")
    save_hf(ours, str(tmp_path / "out"))
    back = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path / "out"), attn_implementation="eager",
                                                             torch_dtype=torch.float32).eval()
    assert type(back).__name__ == ours.args.to_hf_config()["architectures"][0]
    g = torch.Generator().manual_seed(2)
    seqs = [torch.randint(1, 160, (17,), generator=g)]
    torch.testing.assert_close(_hf_logits(back, seqs), _our_logits(ours, seqs), rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("name", ["llama", "mixtral", "qwen2_moe", "olmoe", "gemma"])
def test_family_engine_greedy_matches_model(name, tmp_path):
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    _hf_model(name, tmp_path / "hf")
    m = _ours(tmp_path / "hf")
    eng = RolloutEngine(m.args, EngineWeights.from_model(m, dtype=torch.float32), max_num_seqs=4, max_model_len=128,
                        block_size=16, kv_cache_gb=0.01, use_cuda_graph=False, enable_prefix_caching=False)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1, 160, (n,), generator=g).tolist() for n in (11, 5)]
    for i, p in enumerate(prompts):
        eng.add_request(GenRequest(i, p, SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True, seed=i)))
    outs = {}
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o.output_ids
    for i, p in enumerate(prompts):
        seq = list(p)
        for _ in range(4):
            logits = _our_logits(m, [torch.tensor(seq)])
            seq.append(int(logits[-1].argmax()))
        assert outs[i] == seq[len(p):], (name, i)
