"""The whole engine on one GPU against the float32 model oracle, for the attention shapes of the
model families the reference serves: GQA groups of 7 (Qwen2-0.5B, head_dim 64, QKV bias),
3 (Llama-3.2-3B, head_dim 128), 5 (Qwen2.5-14B) and 6 (Qwen2.5-1.5B) query heads per KV head,
and a group of 16 (the decode kernel's second MMA row group).

Prefill logits are compared with the oracle's, then every decode step's logits with the oracle
run on the same token sequence (teacher forcing), so bf16 rounding cannot move the comparison
onto a different continuation. Two layers of each shape, a small FFN and vocabulary.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 4


@pytest.mark.parametrize("h,hkv,d,bias", [(14, 2, 64, True), (24, 8, 128, False), (40, 8, 128, True),
                                          (12, 2, 128, True), (32, 2, 64, False)])
def test_engine_gqa_groups_match_oracle(h, hkv, d, bias):
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models import reference_model
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", 0)
    cfg = preset("tiny-gpu")
    cfg.num_heads, cfg.num_kv_heads, cfg.hidden_size = h, hkv, h * d
    cfg.attention_bias = bias
    cfg.rope_theta = 1000000.0
    hf = ModelWeights.random_init(cfg, seed=3, device=dev, dtype=torch.bfloat16)
    w = PreparedWeights.from_weights(hf)
    L = 300
    prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(7))
    eng = LlamaCPEngine(cfg, w, device=dev, max_context=L, max_batch=1, decode_reserve=16)
    tok, logits = eng.prefill(1, prompt, [L], decode_horizon=STEPS + 1, return_logits=True)
    seq = prompt.tolist() + [int(tok)]
    got = [logits.float().cpu()]
    for _ in range(STEPS):
        nxt = eng.decode_step([1], torch.tensor([seq[-1]], device=dev))
        got.append(eng.last_logits(1)[0].float().cpu())
        seq.append(int(nxt))
    eng.check_device()
    eng.close()
    for i, g in enumerate(got):
        ids = torch.tensor(seq[:L + i], device=dev)
        ref = reference_model.forward(hf, ids, last_only=True)[0].float().cpu()
        err = (g - ref).abs()
        # bf16 rounding error grows with the logits' scale (std ~ 0.02 sqrt(hidden) here:
        # 0.6 at hidden 896, 1.4 at hidden 5120)
        scale = max(1.0, float(ref.std()))
        assert err.max() < 0.15 * scale and err.mean() < 0.025 * scale, \
            (i, float(err.max()), float(err.mean()), scale)


def test_session_append_matches_oracle():
    """A kept session continued by an appended segment (the keep_kv / append path): prefill,
    decode, append a segment after the last generated token, decode again; every step's logits
    against the oracle on the same token sequence."""
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models import reference_model
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", 0)
    cfg = preset("tiny-gpu")
    hf = ModelWeights.random_init(cfg, seed=5, device=dev, dtype=torch.bfloat16)
    w = PreparedWeights.from_weights(hf)
    g = torch.Generator().manual_seed(9)
    a = torch.randint(0, cfg.vocab_size, (300,), generator=g)
    b = torch.randint(0, cfg.vocab_size, (150,), generator=g).tolist()
    eng = LlamaCPEngine(cfg, w, device=dev, max_context=1024, max_batch=1, decode_reserve=64)
    tok, lg = eng.prefill(3, a, [300], decode_horizon=4, keep_kv=True, return_logits=True)
    seq = a.tolist() + [int(tok)]
    got = [(len(seq) - 1, lg.float().cpu())]
    for _ in range(3):
        nxt = eng.decode_step([3], torch.tensor([seq[-1]], device=dev))
        got.append((len(seq), eng.last_logits(1)[0].float().cpu()))
        seq.append(int(nxt))
    L0 = eng.reqs[3].context_len
    seg = [seq[-1]] + b
    tok2, lg2 = eng.append(3, torch.tensor(seg), list(range(L0, L0 + len(seg))), [1],
                           return_logits=True)
    seq = seq + b
    got.append((len(seq), lg2.float().cpu()))
    seq.append(int(tok2))
    for _ in range(2):
        nxt = eng.decode_step([3], torch.tensor([seq[-1]], device=dev))
        got.append((len(seq), eng.last_logits(1)[0].float().cpu()))
        seq.append(int(nxt))
    eng.check_device()
    eng.close()
    for n, lgt in got:
        ref = reference_model.forward(hf, torch.tensor(seq[:n], device=dev), last_only=True)[0]
        err = (lgt - ref.float().cpu()).abs()
        assert err.max() < 0.15 and err.mean() < 0.02, (n, float(err.max()), float(err.mean()))


@pytest.mark.parametrize("env_kwargs", [dict(decode_prefetch=1), dict(decode_prefetch=3),
                                        dict(decode_splits=8), dict(decode_combine="gemv"),
                                        dict(decode_chain=True)])
def test_decode_switches_keep_the_tokens(env_kwargs):
    """Decode switches that only move work around (L2 prefetch of later weights, a cap on the
    KV splits, where the cross-rank combine runs: unused on one rank, the GEMVs between two
    attentions as one chain launch instead of four launches) give the default engine's greedy
    tokens; the split cap changes the attention's summation order, so its logits are held to the
    bf16 tolerance instead of bit equality."""
    from hetero_cp_ringattn_b200.config import EnvConfig, preset
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", 0)
    cfg = preset("tiny-gpu")
    hf = ModelWeights.random_init(cfg, seed=5, device=dev, dtype=torch.bfloat16)
    w = PreparedWeights.from_weights(hf)
    L = 2000
    prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(9))

    def run(env):
        eng = LlamaCPEngine(cfg, w, device=dev, max_context=L, max_batch=1, decode_reserve=16, env=env)
        tok, _ = eng.prefill(1, prompt, [L], decode_horizon=8)
        toks, logits, cur = [int(tok)], [], tok
        for _ in range(6):
            cur = eng.decode_step([1], cur)
            toks.append(int(cur))
            logits.append(eng.last_logits(1)[0].float().cpu())
        eng.check_device()
        eng.release(1)
        eng.close()
        return toks, torch.stack(logits)

    base_t, base_l = run(EnvConfig())
    got_t, got_l = run(EnvConfig(**env_kwargs))
    if "decode_splits" in env_kwargs:
        assert (got_l - base_l).abs().max() < 0.1 * max(1.0, float(base_l.std()))
    else:
        assert torch.equal(got_l, base_l)
        assert got_t == base_t


def test_long_context_prefill_64k_matches_oracle():
    """A 65,536-token prefill through the engine (two layers of the Llama-3.2-1B shape) and one
    decode step against the float32 oracle, whose attention runs in query chunks at this
    length: the long-context path end to end on one GPU (KV pages, staging buffers of 64k
    positions, 512 KV tiles per q tile at the end of the prompt, decode over 64k cached rows)."""
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models import reference_model
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", 0)
    cfg = preset("llama-3.2-1b")
    cfg.num_layers = 2
    hf = ModelWeights.random_init(cfg, seed=8, device=dev, dtype=torch.bfloat16)
    w = PreparedWeights.from_weights(hf)
    L = 65536
    prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(12))
    eng = LlamaCPEngine(cfg, w, device=dev, max_context=L, max_batch=1, decode_reserve=16)
    tok, logits = eng.prefill(1, prompt, [L], decode_horizon=4, return_logits=True)
    nxt = eng.decode_step([1], tok)
    dec_logits = eng.last_logits(1)[0].float().cpu()
    eng.check_device()
    eng.release(1)
    eng.close()
    seq = torch.cat([prompt.to(dev), tok.view(1).to(dev)])
    for i, got in enumerate((logits.float().cpu(), dec_logits)):
        ref = reference_model.forward(hf, seq[:L + i], last_only=True)[0].float().cpu()
        err = (got - ref).abs()
        scale = max(1.0, float(ref.std()))
        assert err.max() < 0.15 * scale and err.mean() < 0.025 * scale, (i, float(err.max()))
    assert int(nxt) >= 0
