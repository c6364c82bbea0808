"""The attention-backend interface (models/attention.py): the engine's prefill and continuation
layers go through `engine.attn`, a backend can be plugged in, and `set_strategy` sets the
default layout.

Parity: rust/src/model/attention/backend.rs:20-80 (`AttentionBackend` with `forward`,
`set_distributed`, `set_strategy`; `LocalAttentionBackend`).
"""

import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.models import reference_model
from hetero_cp_ringattn_b200.models.attention import (AttentionBackend, HostRingBackend,
                                                      LayerCall)
from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
from hetero_cp_ringattn_b200.ops import reference as ref
from hetero_cp_ringattn_b200.parallel.strategy import RingStrategy


def _weights():
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=4, dtype=torch.float32, std=0.2)
    return cfg, w, PreparedWeights.from_weights(w, dtype=torch.float32)


class DenseLocalBackend(AttentionBackend):
    """A backend written against the interface alone: one rank, dense causal attention over the
    rows it has stored so far (the reference's local GQA backend)."""

    name = "dense_local"

    def __init__(self, eng):
        super().__init__(eng)
        self.calls = 0

    def forward(self, xn, lw, call: LayerCall):
        e, cfg = self.eng, self.eng.cfg
        self.calls += 1
        T = int(call.pos.numel())
        H, Hkv, D = e.H, e.Hkv, e.D
        qkv = ref.linear(xn, lw.wqkv, lw.bqkv)
        q = ref.apply_rope(qkv[:, :H * D].view(T, H, D), call.pos, cfg.rope_theta, cfg.rope_scaling)
        k = ref.apply_rope(qkv[:, H * D:(H + Hkv) * D].view(T, Hkv, D), call.pos, cfg.rope_theta,
                           cfg.rope_scaling)
        v = qkv[:, (H + Hkv) * D:].reshape(T, Hkv, D)
        if call.existing is None:
            call.st.host_kv.append([k, v, call.pos.clone(), torch.ones(T, dtype=torch.bool)])
        else:
            kv = call.st.host_kv[call.layer]
            kv[0], kv[1] = torch.cat([kv[0], k]), torch.cat([kv[1], v])
            kv[2] = torch.cat([kv[2], call.pos])
            kv[3] = torch.cat([kv[3], torch.ones(T, dtype=torch.bool)])
        kv = call.st.host_kv[call.layer]
        o, _ = ref.full_attention(q, kv[0], kv[1], call.pos, kv[2], causal=True)
        return o.reshape(T, H * D)


def test_default_backend_and_plugged_in_backend_agree():
    cfg, w, pw = _weights()
    prompt = torch.randint(0, cfg.vocab_size, (41,), generator=torch.Generator().manual_seed(6))
    seg = torch.randint(0, cfg.vocab_size, (9,), generator=torch.Generator().manual_seed(7))
    out = {}
    for name, backend in (("host", None), ("dense", DenseLocalBackend)):
        eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=256,
                            attention_backend=backend)
        assert eng.attn.mode == "local"
        tok, logits = eng.prefill(1, prompt, [41], decode_horizon=8, keep_kv=True, return_logits=True)
        nxt, cont = eng.append(1, seg, list(range(41, 50)), [1], return_logits=True)
        out[name] = (logits, cont, eng.attn)
    assert isinstance(out["host"][2], HostRingBackend)
    assert out["dense"][2].calls == 2 * cfg.num_layers      # prefill + continuation, every layer
    want = reference_model.forward(w, prompt, last_only=True)[0]
    for name in out:
        assert (out[name][0] - want).abs().max() < 1e-4, name
    assert (out["host"][1] - out["dense"][1]).abs().max() < 1e-4
    want_cont = reference_model.forward(w, torch.cat([prompt, seg]), last_only=True)[0]
    assert (out["dense"][1] - want_cont).abs().max() < 1e-4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _strategy_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w, pw = _weights()
        eng = LlamaCPEngine(cfg, pw, rank=rank, world=world, device=torch.device("cpu"),
                            group=dist.group.WORLD, max_context=256)
        assert eng.attn.mode == "ring"
        eng.attn.set_strategy("zigzag")
        prompt = torch.randint(0, cfg.vocab_size, (48,), generator=torch.Generator().manual_seed(8))
        _, logits = eng.prefill(3, prompt, [24, 24], decode_horizon=4, return_logits=True)
        assert eng.reqs[3].strategy == RingStrategy.ZIGZAG
        if rank == 0:
            want = reference_model.forward(w, prompt, last_only=True)[0]
            torch.save(float((logits - want).abs().max()), out)
        dist.barrier()   # neither rank tears the group down while the other still uses it
    finally:
        dist.destroy_process_group()


def test_set_strategy_sets_the_default_layout_on_two_ranks():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "r.pt")
        mp.start_processes(_strategy_worker, args=(2, _port(), out), nprocs=2, join=True,
                           start_method="spawn")
        assert torch.load(out) < 1e-4
