"""Same-box comparator: a PyTorch restatement of the reference's inference algorithm.

This is NOT the reference (stark-sim/hetero-cp-ringattn is a Rust/tch-rs program that cannot be
built here; see bench.py --impl reference). It restates the reference's algorithm with stock
PyTorch ops on the same GPUs so the framework's kernels can be compared against "the reference's
approach on libtorch + cuBLAS + NCCL":

  * projections, norms, RoPE, SwiGLU: torch ops / F.linear (cuBLAS), bf16, HF layout
    (rust/src/model/layers/{norm,rotary,mlp,attention}.rs);
  * ring attention (rust/src/model/attention/ring.rs:861-1399): local Q split into q-chunks of
    clamp(ceil(L_loc / N), 1, 2048) rows, KV split into micro-blocks of max(kv_chunk, 1024)
    tokens, K/V expanded to all query heads before use (ring.rs:1962-1984), score blocks
    [H, qc, kc] materialised per block, fully-future blocks skipped, online (m, l, O) update;
    blocks travel around the ring with NCCL send/recv as float32 (the reference's wire format,
    quic.rs:935-937), N-1 rounds per layer;
  * decode: the (Q, O, LSE) accumulator ring (ring.rs:682-818) - every rank computes its local
    partial, partials move N-1 hops around the ring and are merged; decode KV is sharded by
    position % N (cache.rs:40-49);
  * first token / greedy decode: LM head on the rank holding the last position, broadcast.
"""

from __future__ import annotations

import math
from typing import List, Sequence

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _rms(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(x.dtype)


def _rope(x, cos, sin):
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return x * cos + torch.cat([-x2, x1], dim=-1) * sin


class RefRingModel:
    def __init__(self, cfg, w: dict, rank: int = 0, world: int = 1, device=None):
        self.cfg, self.w, self.rank, self.world = cfg, w, rank, world
        self.dev = device
        self.H, self.Hkv, self.D = cfg.num_heads, cfg.kv_heads, cfg.head_dim
        self.scale = 1.0 / math.sqrt(self.D)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, self.D, 2, device=device).float() / self.D))
        self.inv_freq = inv
        self.cache: List[list] = []

    def _cos_sin(self, pos):
        f = pos.float()[:, None] * self.inv_freq[None]
        emb = torch.cat([f, f], dim=-1)
        return emb.cos().to(torch.bfloat16)[:, None], emb.sin().to(torch.bfloat16)[:, None]

    def _expand(self, t):
        return t.repeat_interleave(self.H // self.Hkv, dim=1)  # materialised GQA expansion

    # ------------------------------------------------------------------ ring attention
    def _block(self, q, k, v, qp, kp, st):
        m, l, acc = st
        if int(kp.min()) > int(qp.max()):
            return st  # fully-future block
        s = torch.einsum("qhd,khd->hqk", q, k) * self.scale          # [H, qc, kc] input dtype
        s = s.float().masked_fill(kp[None, None, :] > qp[None, :, None], float("-inf"))
        mb = s.amax(-1)
        mn = torch.maximum(m, mb)
        a = torch.exp(m - mn)
        p = torch.exp(s - mn[..., None])
        l = l * a + p.sum(-1)
        acc = acc * a.transpose(0, 1)[..., None] + torch.einsum("hqk,khd->qhd", p.to(v.dtype), v).float()
        return mn, l, acc

    def _ring_attention(self, q, k, v, pos):
        N, r = self.world, self.rank
        Lloc = q.shape[0]
        qc = max(1, min(2048, -(-Lloc // N)))
        micro = max(qc, 1024)
        ke, ve = self._expand(k), self._expand(v)
        states = []
        for a in range(0, Lloc, qc):
            b = min(Lloc, a + qc)
            states.append((torch.full((self.H, b - a), -1e4, device=self.dev),
                           torch.zeros(self.H, b - a, device=self.dev),
                           torch.zeros(b - a, self.H, self.D, device=self.dev), a, b))

        def fold(kk, vv, kp):
            for i, (m, l, acc, a, b) in enumerate(states):
                for c in range(0, kk.shape[0], micro):
                    d = min(kk.shape[0], c + micro)
                    m, l, acc = self._block(q[a:b], kk[c:d], vv[c:d], pos[a:b], kp[c:d], (m, l, acc))
                states[i] = (m, l, acc, a, b)

        fold(ke, ve, pos)
        if N > 1:
            # rotate float32 blocks around the ring: N - 1 rounds
            blk_k, blk_v, blk_p = ke.float(), ve.float(), pos.clone()
            sizes = [torch.zeros(1, dtype=torch.int64, device=self.dev) for _ in range(N)]
            dist.all_gather(sizes, torch.tensor([Lloc], device=self.dev))
            for rnd in range(1, N):
                src = (r - rnd) % N
                n_in = int(sizes[src])
                rk = torch.empty(n_in, self.H, self.D, device=self.dev)
                rv = torch.empty_like(rk)
                rp = torch.empty(n_in, dtype=pos.dtype, device=self.dev)
                ops = [dist.P2POp(dist.isend, blk_k, (r + 1) % N), dist.P2POp(dist.irecv, rk, (r - 1) % N),
                       dist.P2POp(dist.isend, blk_v, (r + 1) % N), dist.P2POp(dist.irecv, rv, (r - 1) % N),
                       dist.P2POp(dist.isend, blk_p, (r + 1) % N), dist.P2POp(dist.irecv, rp, (r - 1) % N)]
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
                fold(rk.to(torch.bfloat16), rv.to(torch.bfloat16), rp)
                blk_k, blk_v, blk_p = rk, rv, rp
        outs = []
        for m, l, acc, a, b in states:
            outs.append((acc / l.transpose(0, 1)[..., None].clamp_min(1e-30)).to(torch.bfloat16))
        return torch.cat(outs)

    # ------------------------------------------------------------------ model
    def _layer_qkv(self, i, x, pos):
        p = f"model.layers.{i}."
        w = self.w
        h = _rms(x, w[p + "input_layernorm.weight"], self.cfg.rms_norm_eps)
        bias = (lambda n: w.get(p + f"self_attn.{n}_proj.bias"))
        q = F.linear(h, w[p + "self_attn.q_proj.weight"], bias("q")).view(-1, self.H, self.D)
        k = F.linear(h, w[p + "self_attn.k_proj.weight"], bias("k")).view(-1, self.Hkv, self.D)
        v = F.linear(h, w[p + "self_attn.v_proj.weight"], bias("v")).view(-1, self.Hkv, self.D)
        cos, sin = self._cos_sin(pos)
        return _rope(q, cos, sin), _rope(k, cos, sin), v

    def _layer_rest(self, i, x, o):
        p = f"model.layers.{i}."
        w = self.w
        x = x + F.linear(o.reshape(o.shape[0], -1), w[p + "self_attn.o_proj.weight"])
        h = _rms(x, w[p + "post_attention_layernorm.weight"], self.cfg.rms_norm_eps)
        g = F.linear(h, w[p + "mlp.gate_proj.weight"])
        u = F.linear(h, w[p + "mlp.up_proj.weight"])
        return x + F.linear(F.silu(g) * u, w[p + "mlp.down_proj.weight"])

    def _logits(self, x):
        h = _rms(x, self.w["model.norm.weight"], self.cfg.rms_norm_eps)
        return F.linear(h, self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])).float()

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, chunks: Sequence[int]) -> torch.Tensor:
        off = sum(chunks[: self.rank])
        T = chunks[self.rank]
        pos = torch.arange(off, off + T, device=self.dev)
        x = self.w["model.embed_tokens.weight"][prompt[off:off + T].to(self.dev)]
        self.cache = []
        for i in range(self.cfg.num_layers):
            q, k, v = self._layer_qkv(i, x, pos)
            self.cache.append([k, v, pos])
            x = self._layer_rest(i, x, self._ring_attention(q, k, v, pos))
        tok = torch.zeros(1, dtype=torch.int64, device=self.dev)
        last = len(chunks) - 1
        if self.rank == last:
            tok[0] = self._logits(x[-1:]).argmax(-1)[0]
        if self.world > 1:
            dist.broadcast(tok, src=last)
        self.next_pos = sum(chunks)
        return tok

    def _qring(self, q, k_loc, v_loc, p_loc):
        ke, ve = self._expand(k_loc), self._expand(v_loc)
        s = torch.einsum("qhd,khd->hqk", q, ke).float() * self.scale
        lse = torch.logsumexp(s, -1)                                  # [H, 1]
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1).to(ve.dtype), ve).float()
        if self.world == 1:
            return o.to(torch.bfloat16)
        N, r = self.world, self.rank
        acc_o, acc_l = o, lse
        pkt_o, pkt_l = o.clone(), lse.clone()
        for _ in range(N - 1):
            ro, rl = torch.empty_like(pkt_o), torch.empty_like(pkt_l)
            ops = [dist.P2POp(dist.isend, pkt_o, (r + 1) % N), dist.P2POp(dist.irecv, ro, (r - 1) % N),
                   dist.P2POp(dist.isend, pkt_l, (r + 1) % N), dist.P2POp(dist.irecv, rl, (r - 1) % N)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            m = torch.maximum(acc_l, rl)
            wa, wb = torch.exp(acc_l - m), torch.exp(rl - m)
            acc_o = (acc_o * wa.transpose(0, 1)[..., None] + ro * wb.transpose(0, 1)[..., None]) / \
                (wa + wb).transpose(0, 1)[..., None]
            acc_l = m + torch.log(wa + wb)
            pkt_o, pkt_l = ro, rl
        return acc_o.to(torch.bfloat16)

    @torch.no_grad()
    def decode_step(self, tok: torch.Tensor) -> torch.Tensor:
        pos = torch.tensor([self.next_pos], device=self.dev)
        x = self.w["model.embed_tokens.weight"][tok.view(1)]
        keep = (self.next_pos % self.world) == self.rank
        for i in range(self.cfg.num_layers):
            q, k, v = self._layer_qkv(i, x, pos)
            c = self.cache[i]
            if keep:
                c[0] = torch.cat([c[0], k])
                c[1] = torch.cat([c[1], v])
                c[2] = torch.cat([c[2], pos])
            x = self._layer_rest(i, x, self._qring(q, c[0], c[1], c[2]))
        self.next_pos += 1
        return self._logits(x).argmax(-1)


def hf_random_weights(cfg, device, seed=0, std=0.02) -> dict:
    """Random-init weights in HF layout (same distribution as the framework's benchmark)."""
    from hetero_cp_ringattn_b200.models.weights import ModelWeights
    return ModelWeights.random_init(cfg, seed=seed, device=device, dtype=torch.bfloat16, std=std).tensors
