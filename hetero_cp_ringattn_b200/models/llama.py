"""Llama / Qwen2 context-parallel inference engine: one instance per rank (one process per GPU).

Parity (reference call stacks):
  * prefill: rust/src/model/model.rs:195-343 (`LlamaModel::forward`), layers/mod.rs:59-90,
    attention/ring.rs:1841-2028 (QKV -> RoPE -> KV cache update -> ring attention -> O proj),
    worker_sdk/tch_backend.rs:126-236 (`do_prefill`, last-token logits on the rank holding the
    final position);
  * decode: the Q-ring / self-driving routes (ring.rs:682-818, self_driving.rs:333-675,
    tch_backend.rs:634-904) with KV growth placed by `FrozenKvAssigneeSchedule`
    (self_driving.rs:12-120), or by global position % N (ring.rs:1934) when
    HCP_RING_DECODE_SD=0; here every rank computes the token's layer in parallel, attends
    over its own shard and combines (O, LSE) with the other ranks inside the decode kernels;
  * HCP_RING_DECODE_RING=0 selects the legacy route (ring.rs:982-997): every rank keeps every
    decoded row and the prefill partitions are re-sent each step. It is a correctness fallback
    of the host path only; CUDA ranks keep the (O, LSE) exchange;
  * release: tch_backend.rs:1077 (`release_request`).

Hot path (CUDA): embedding, RMSNorm, tcgen05 GEMMs with fused bias / residual / SwiGLU epilogues,
the runtime's fused RoPE + KV write + NVLink push and ring attention (prefill), weight-streaming
GEMVs, KV append, split-KV attention with the in-kernel cross-rank (O, LSE) exchange, and the
LM-head GEMV with a fused argmax (decode). The decode step is captured in a CUDA graph.

Host path (CPU tensors, gloo process group): the same algorithm with the plain PyTorch oracles
and torch.distributed all-gathers standing in for the NVLink exchange. It exists for CPU-rank
tests of the distributed logic; it is never used when the engine runs on a GPU.
"""

from __future__ import annotations

import dataclasses
import math
import time
import warnings
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist

from ..config import EnvConfig, ModelConfig
from ..errors import CapacityError, RingError
from ..kv.arena import KvArenaManager, RequestKv
from ..ops import kernels as K
from ..ops import reference as ref
from ..ops._ext import native
from ..parallel.schedule import assignee_table
from ..parallel.strategy import RingStrategy, build_assignment, build_domain_positions
from ..utils import launches
from ..utils.perf import PerfLog, peak_bf16_tflops
from .attention import AttentionBackend, LayerCall, default_backend, positions_tensor
from .weights import PreparedWeights


def ring_plan(positions: Sequence[np.ndarray], rank: int, L: int, tile: int = 128):
    """Host plan of the overlapped in-kernel ring for one request (the same for every layer).

    positions[r] are rank r's global prompt positions (ascending, any layout). Returns
      tile_src   int64 [ceil(L / tile)]: bit r set when rank r holds rows of KV tile t (the
                 attention waits for the flags of exactly these (tile, rank) pairs);
      push_tiles int32 [n, 3]: this rank's own tiles as (tile, first row, end row) ranges of its
                 positions, last tile first (the order in which its kernel pushes them).
    """
    ntiles = -(-int(L) // tile)
    src = np.zeros(ntiles, dtype=np.uint64)
    for r, p in enumerate(positions):
        if len(p):
            src[np.unique(np.asarray(p, dtype=np.int64) // tile)] |= np.uint64(1) << np.uint64(r)
    own = np.asarray(positions[rank], dtype=np.int64)
    if len(own) == 0:
        return src.view(np.int64), np.zeros((0, 3), dtype=np.int32)
    if np.any(np.diff(own) <= 0):
        raise RingError("ring plan: a rank's positions must be strictly increasing")
    tiles, lo = np.unique(own // tile, return_index=True)
    hi = np.r_[lo[1:], len(own)]
    push = np.stack([tiles, lo, hi], 1)[::-1].astype(np.int32)
    return src.view(np.int64), np.ascontiguousarray(push)


@dataclasses.dataclass
class RequestState:
    req_id: int
    prompt_len: int
    chunks: list
    strategy: RingStrategy
    positions: np.ndarray            # this rank's prompt positions (local order)
    owner_of_last: int
    horizon: int
    assignee: np.ndarray             # [horizon, layers] rank storing (token, layer) KV
    decode_offset: int = 0
    context_len: int = 0             # tokens with KV (prompt + decoded)
    kv: Optional[RequestKv] = None
    host_kv: Optional[list] = None   # CPU path: per layer [k [n,Hkv,D], v, pos [n], shared [n]]
                                     # shared: the row lives on this rank only (prompt / segment /
                                     # owned growth); False: a replicated legacy-decode row
    keep_kv: bool = False
    ring: Optional[tuple] = None     # device tensors of ring_plan (overlapped CUDA ring only)


class LlamaCPEngine:
    def __init__(self, cfg: ModelConfig, weights: PreparedWeights, *, rank: int = 0,
                 world: int = 1, device: Optional[torch.device] = None,
                 group: Optional["dist.ProcessGroup"] = None, max_context: int = 8192,
                 max_batch: int = 8, page_size: Optional[int] = None, kv_pages: Optional[int] = None,
                 decode_reserve: int = 512, env: Optional[EnvConfig] = None,
                 use_graphs: bool = True, perf_log: Optional[PerfLog] = None,
                 attention_backend=None):
        cfg.validate()
        self.cfg = cfg
        self.w = weights
        self.rank = rank
        self.world = world
        self.group = group
        self.env = env or EnvConfig.from_env()
        self.device = device or weights.embed.device
        self.cuda = self.device.type == "cuda"
        self.max_context = int(max_context)
        self.max_batch = int(max_batch)
        if self.cuda and not 1 <= self.max_batch <= 8:
            raise CapacityError(f"max_batch {self.max_batch}: the CUDA decode step batches 1 to 8 "
                                "requests (graph buckets 1, 2, 4, 8)")
        # tokens per KV page: HCP_KV_CACHE_BLOCK_SIZE unless given; the arena is always paged
        # (HCP_KV_CACHE_BLOCK_TABLE has nothing to switch off)
        self.page_size = int(page_size if page_size is not None else self.env.kv_block_size)
        if self.page_size <= 0 or (self.cuda and self.page_size % 128):
            raise CapacityError(f"KV page size {self.page_size} must be a positive multiple of 128 "
                                f"tokens on CUDA (the attention kernels read 128-token tiles)")
        # host-path ring fold granularity (HCP_MICRO_KV_BLOCK_SIZE; 0 -> the CUDA tile, 128).
        # The CUDA kernels always stream 128-token KV tiles.
        self.micro_kv = int(self.env.micro_kv_block_size) or 128
        self.legacy_decode = not self.env.decode_ring
        if self.legacy_decode and self.cuda:
            warnings.warn("HCP_RING_DECODE_RING=0 (legacy KV re-send decode) is a host-path "
                          "correctness fallback; CUDA ranks decode with the (O, LSE) exchange",
                          RuntimeWarning, stacklevel=2)
            self.legacy_decode = False
        self.H, self.Hkv, self.D = cfg.num_heads, cfg.kv_heads, cfg.head_dim
        self.L = cfg.num_layers
        self.scale = 1.0 / math.sqrt(self.D)
        self.use_graphs = use_graphs and self.cuda
        self.perf = perf_log or PerfLog.from_env(self.env)
        # overlapped ring: the attention kernel pushes this rank's K/V rows to the peers and waits
        # per tile; serial ring: push everything, wait for every rank, then attend. Measured on
        # B200 (Llama-3.2-1B shape, 32k): overlapped is faster on 2 ranks (TTFT 76.4 vs 77.5 ms),
        # serial on 8 (22.98 vs 23.91 ms: each rank pushes 58 MB, and the first CTAs run out of
        # own tiles long before two pusher warps per SM have delivered the remote ones), so the
        # default switches at 3 ranks; HCP_DISABLE_OVERLAP=1 / =0 (the reference's switch) forces
        # the serial / overlapped ring
        if self.env.disable_overlap is None:
            self.overlap = 1 < world <= 2
        else:
            self.overlap = world > 1 and not self.env.disable_overlap
        # fused QKV projection (RoPE + Q / arena / staging writes in the GEMM epilogue): faster on
        # one rank (+2% prefill) and in the overlapped ring, where the epilogue writes only the
        # local staging buffer; the serial ring keeps the separate push kernel, which spreads the
        # peer stores over every SM's threads instead of the epilogue's 4 warps (1.05M vs 1.22M
        # prefill tok/s at CP=8). An explicit HCP_FUSED_QKV overrides.
        self.fused_qkv = (self.env.fused_qkv if self.env.fused_qkv is not None
                          else (world == 1 or self.overlap))
        self.fused_qkv_serial = self.env.fused_qkv if self.env.fused_qkv is not None else world == 1
        self.tok_epoch = 0
        # prefill / continuation attention (models/attention.py): an AttentionBackend instance,
        # or a class taking the engine; default: the CUDA ring on GPUs, the host ring on CPU
        if isinstance(attention_backend, type):
            attention_backend = attention_backend(self)
        self.attn: AttentionBackend = attention_backend or default_backend(self)
        if kv_pages is None:
            kv_pages = -(-self.max_context // self.page_size) + \
                max_batch * -(-decode_reserve // self.page_size) + 2
        self.kv = KvArenaManager(kv_pages, self.page_size, self.L)
        max_pos = self.max_context + max(decode_reserve, 1) + 8
        cos, sin = ref.rope_cos_sin(torch.arange(max_pos, device=self.device), self.D, cfg.rope_theta,
                                       scaling=cfg.rope_scaling)
        self.cos, self.sin = cos.contiguous(), sin.contiguous()
        self.reqs: Dict[int, RequestState] = {}
        self.prefill_epoch = 0
        self.rt = None
        if self.cuda:
            self.rt = native().Runtime(rank, world, self.device.index or 0, self.L, kv_pages,
                                       self.page_size, self.Hkv, self.D, self.H,
                                       self.max_context, self.max_batch,
                                       self.env.p2p_spin_budget_ms)
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, self.rt.export_handle(), group=group)
                self.rt.open_peers(handles)
                dist.barrier(group=group)
            self.dec_step = torch.zeros(1, dtype=torch.int64, device=self.device)
            self._graphs: Dict[int, "DecodeGraph"] = {}
            self._last_split = False
            self.num_sms = native().num_sms(self.device.index or 0)
            # greedy decode on several ranks: rank r runs the LM head over vocabulary rows
            # [vocab_lo, vocab_hi) only and the ranks exchange their packed argmax (the token is
            # the whole head's argmax, ties to the smaller id); steps that need logits run the
            # whole head on every rank
            V = cfg.vocab_size
            part = -(-V // (world * 8)) * 8
            self.vocab_lo = min(V, rank * part)
            self.vocab_hi = min(V, self.vocab_lo + part)
            self.split_head = world > 1 and self.env.split_lm_head and V - (world - 1) * part > 0
            self.lm_head_slice = self.w.lm_head[self.vocab_lo:self.vocab_hi]

    # ------------------------------------------------------------------ helpers
    def kv_capacity_bytes(self) -> Optional[int]:
        """Bytes of this rank's preallocated KV arena (bf16 K and V, every layer); None on the
        host path, whose KV lives in ordinary tensors."""
        if not self.cuda:
            return None
        return int(self.kv.alloc.num_pages * self.page_size * self.L *
                   self.cfg.kv_bytes_per_token_per_layer(2))

    def staging_capacity_bytes(self) -> Optional[int]:
        """Bytes of this rank's prefill KV staging buffers (two parities of position-ordered K
        and V up to `max_context`; the same on every rank, see `kv.arena.staging_bytes`); None
        on the host path."""
        if not self.cuda:
            return None
        from ..kv.arena import staging_bytes
        return staging_bytes(self.max_context, self.Hkv, self.D)

    def close(self, sync: bool = True) -> None:
        """Free the graphs and the runtime. `sync` waits for every rank first (peers may still
        read this rank's region); pass False when the other ranks are stopping as well."""
        self._graphs = {} if self.cuda else None
        if self.rt is not None:
            if sync and self.world > 1 and dist.is_initialized():
                dist.barrier(group=self.group)
            self.rt.shutdown()
            self.rt = None

    def check_device(self) -> None:
        if self.rt is not None:
            self.rt.check()

    def layout(self, chunks: Sequence[int], strategy) -> tuple:
        assignment = build_assignment(chunks, strategy)
        positions = build_domain_positions(assignment, len(chunks))
        return assignment, positions

    def _schedule(self, req_id: int, tickets: Sequence[int], horizon: int,
                  first_t: int = 0, first_pos: int = 0) -> np.ndarray:
        """[horizon, layers]: the rank that stores each decoded (token, layer) KV row. Row t is
        the request's t-th decoded token; rows before `first_t` are already consumed and the
        token of row `first_t` sits at global position `first_pos`."""
        if horizon <= 0:
            return np.zeros((0, self.L), dtype=np.int64)
        if not self.env.decode_sd:
            # Q-ring placement (ring.rs:1934): position p is kept by rank p % N on every layer
            owners = (first_pos + np.arange(horizon, dtype=np.int64) - first_t) % self.world
            return np.repeat(owners[:, None], self.L, axis=1)
        return assignee_table(tickets, req_id, horizon, self.L)

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, req_id: int, prompt_ids: torch.Tensor, chunks: Sequence[int],
                strategy=None, decode_horizon: int = 128,
                tickets: Optional[Sequence[int]] = None, return_logits: bool = False,
                keep_kv: bool = False):
        """SPMD prefill of one request. Every rank passes the same full prompt and chunk split.

        Returns (first_token: int64 device tensor [1], logits or None). The first token is
        broadcast from the rank holding the last prompt position. `strategy` None: the attention
        backend's default layout (`self.attn.set_strategy`, vanilla unless set)."""
        strategy = RingStrategy.parse(strategy if strategy is not None else self.attn.strategy)
        chunks = [int(c) for c in chunks]
        if len(chunks) != self.world:
            raise RingError(f"{len(chunks)} chunks for {self.world} ranks")
        Lp = sum(chunks)
        if Lp + decode_horizon > self.cos.shape[0] or Lp > self.max_context:
            raise CapacityError(f"prompt {Lp} (+{decode_horizon}) exceeds the engine's context "
                                f"capacity {self.max_context}")
        if self.cfg.max_position_embeddings and Lp + decode_horizon > self.cfg.max_position_embeddings:
            raise CapacityError(f"prompt {Lp} + {decode_horizon} exceeds max_position_embeddings "
                                f"{self.cfg.max_position_embeddings}")
        if req_id in self.reqs:
            raise RingError(f"request {req_id} already active on rank {self.rank}")
        assignment, positions = self.layout(chunks, strategy)
        my_pos = positions[self.rank]
        T = len(my_pos)
        tickets = list(tickets) if tickets is not None else list(chunks)
        assignee = self._schedule(req_id, tickets, decode_horizon, 0, Lp)
        growth = int((assignee == self.rank).sum(0).max()) if decode_horizon else 0
        st = RequestState(req_id=req_id, prompt_len=Lp, chunks=chunks, strategy=strategy,
                          positions=my_pos, owner_of_last=int(assignment[Lp - 1]),
                          horizon=decode_horizon, assignee=assignee, context_len=Lp,
                          keep_kv=keep_kv)
        t0 = time.perf_counter()
        if self.cuda:
            st.kv = self.kv.reserve(req_id, T, T + growth, my_pos)
            st.kv.pt_device = torch.tensor(st.kv.pages, dtype=torch.int32, device=self.device)
            if self.overlap:
                plan = ring_plan(positions, self.rank, Lp)
                st.ring = tuple(torch.from_numpy(x).to(self.device) for x in plan)
            ids_local = prompt_ids.to(self.device, non_blocking=True)[torch.from_numpy(my_pos).to(self.device)]
            tok, logits = self._prefill_cuda(st, ids_local.int(), Lp, return_logits)
        else:
            ids_local = prompt_ids[torch.from_numpy(my_pos)]
            tok, logits = self._prefill_host(st, ids_local, Lp, return_logits)
        self.reqs[req_id] = st
        if self.perf.enabled:
            self.perf.emit("prefill", rank=self.rank, request=req_id, tokens=T, prompt=Lp,
                           host_ms=(time.perf_counter() - t0) * 1e3, world=self.world)
        return tok, logits

    def _prefill_cuda(self, st: RequestState, ids: torch.Tensor, Lp: int, return_logits: bool):
        w, dev = self.w, self.device
        T = ids.numel()
        pos = positions_tensor(st.positions, dev)
        x = K.embedding(ids, w.embed)
        xn = torch.empty_like(x)
        q_buf = torch.empty(T, self.H, self.D, dtype=torch.bfloat16, device=dev)
        o_buf = torch.empty_like(q_buf)
        ring = {}
        if st.ring is not None:
            ring = dict(tile_src=st.ring[0], push_tiles=st.ring[1])
        trace = self.perf.enabled
        nvtx = self.env.nvtx
        for li, lw in enumerate(w.layers):
            if nvtx:
                torch.cuda.nvtx.range_push(f"prefill layer {li}")
            if trace:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
                ev[0].record()
            K.rmsnorm(x, lw.in_norm, self.cfg.rms_norm_eps, out=xn)
            self.prefill_epoch += 1
            if trace:
                ev[1].record()
            o = self.attn.forward(xn, lw, LayerCall(st, li, pos, Lp, q_buf, o_buf, self.prefill_epoch,
                                                    ring=ring, ev=ev if trace else None))
            if trace:
                ev[3].record()
            K.gemm(o, lw.wo, "residual", residual=x)
            K.rmsnorm(x, lw.post_norm, self.cfg.rms_norm_eps, out=xn)
            g = K.gemm(xn, lw.wgu, "swiglu")
            K.gemm(g, lw.wd, "residual", residual=x)
            del g
            if trace:
                ev[4].record()
                self._emit_layer(st, li, T, Lp, ev)
            if nvtx:
                torch.cuda.nvtx.range_pop()
        return self._first_token_cuda(st, x, return_logits)

    def _emit_layer(self, st: RequestState, layer: int, T: int, Lp: int, ev) -> None:
        """`ring_attention` perf event (the reference's HCP_PERF_LOG schema, ring.rs:1376-1395),
        device-timed with CUDA events; bytes are the bf16 compact-GQA K/V rows this rank pushed to
        its peers over NVLink and the rows its peers pushed to it."""
        ev[4].synchronize()
        row_bytes = 2 * self.Hkv * self.D * 2
        sent = T * row_bytes * (self.world - 1)
        recv = (Lp - T) * row_bytes
        attn_ms = ev[2].elapsed_time(ev[3])
        proj_ms = ev[1].elapsed_time(ev[2])
        tflops = 4.0 * self.H * self.D * float(np.sum(st.positions + 1)) / max(attn_ms, 1e-6) / 1e9
        overlap = self.overlap and st.ring is not None
        # overlapped ring: the push runs inside the attention kernel, so the attention interval
        # holds local compute, peer compute and the push, and the NVLink rate is averaged over it;
        # serial ring: the push (and its waits) sit between the projection and the attention
        span_ms = attn_ms if overlap else proj_ms
        self.perf.emit("ring_attention", domain=self.rank, layer=layer, request=st.req_id,
                       total_ms=ev[0].elapsed_time(ev[4]), qkv_ms=ev[0].elapsed_time(ev[1]),
                       send_ms=proj_ms, local_compute_ms=attn_ms,
                       peer_compute_ms=None if (overlap or self.world == 1) else 0.0,
                       recv_ms=0.0, forward_ms=0.0, flush_ms=0.0,
                       mlp_ms=ev[3].elapsed_time(ev[4]), kv_sent_bytes=sent, kv_recv_bytes=recv,
                       wire_sent_bytes=sent, wire_recv_bytes=recv, micro_blocks=-(-Lp // 128),
                       num_domains=self.world, seq_len=T, overlap=overlap,
                       ring_mode=("single" if self.world == 1 else
                                  "overlap_in_kernel" if overlap else "serial"),
                       attention_backend=self.attn.name,
                       nvlink_gbps=sent / max(span_ms, 1e-6) / 1e6,
                       nvlink_span="attention" if overlap else "projection+push",
                       attn_tflops=tflops, roofline_frac=tflops / peak_bf16_tflops())

    def _first_token_cuda(self, st: RequestState, x: torch.Tensor, return_logits: bool):
        dev = self.device
        tok = torch.zeros(1, dtype=torch.int64, device=dev)
        logits = None
        if self.rank == st.owner_of_last:
            row = int(np.nonzero(st.positions == st.prompt_len - 1)[0][0])
            xl = torch.empty(1, self.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
            K.rmsnorm(x[row:row + 1], self.w.final_norm, self.cfg.rms_norm_eps, out=xl)
            am = torch.zeros(1, dtype=torch.int64, device=dev)
            logits = torch.empty(1, self.cfg.vocab_size, dtype=torch.float32, device=dev)
            K.gemv(xl, self.w.lm_head, "argmax", y_f32=logits, argmax=am)
            native().argmax_finalize(am, None, tok)
            launches.count()
        if self.world > 1:
            # the token goes from the owner's memory to every rank's token slot over NVLink (a
            # bounded device wait on the others): no host round trip inside the TTFT
            self.tok_epoch += 1
            self.rt.broadcast_token(tok, st.owner_of_last, self.tok_epoch)
            launches.count()
            if return_logits:
                if logits is None:
                    logits = torch.empty(1, self.cfg.vocab_size, dtype=torch.float32, device=dev)
                dist.broadcast(logits, src=st.owner_of_last, group=self.group)
        return tok, (logits[0] if (return_logits and logits is not None) else None)

    # ------------------------------------------------------------------ host (CPU) prefill
    def _gather_rows(self, t: torch.Tensor) -> List[torch.Tensor]:
        if self.world == 1:
            return [t]
        n = torch.tensor([t.shape[0]], dtype=torch.int64)
        sizes = [torch.zeros_like(n) for _ in range(self.world)]
        dist.all_gather(sizes, n, group=self.group)
        mx = int(max(int(s) for s in sizes))
        pad = torch.zeros((mx,) + tuple(t.shape[1:]), dtype=t.dtype)
        pad[: t.shape[0]] = t
        bufs = [torch.zeros_like(pad) for _ in range(self.world)]
        dist.all_gather(bufs, pad, group=self.group)
        return [b[: int(s)] for b, s in zip(bufs, sizes)]

    def _prefill_host(self, st: RequestState, ids: torch.Tensor, Lp: int, return_logits: bool):
        w, cfg = self.w, self.cfg
        pos = positions_tensor(st.positions, self.device)
        x = w.embed[ids.long()].float()
        st.host_kv = []
        for li, lw in enumerate(w.layers):
            h = ref.rmsnorm(x, lw.in_norm, cfg.rms_norm_eps)
            o = self.attn.forward(h, lw, LayerCall(st, li, pos, Lp))
            x = x + ref.linear(o, lw.wo)
            h = ref.rmsnorm(x, lw.post_norm, cfg.rms_norm_eps)
            x = x + ref.linear(K.swiglu_from_interleaved(ref.linear(h, lw.wgu)), lw.wd)
        tok = torch.zeros(1, dtype=torch.int64)
        logits = torch.zeros(cfg.vocab_size, dtype=torch.float32)
        if self.rank == st.owner_of_last:
            row = int(np.nonzero(st.positions == Lp - 1)[0][0])
            xl = ref.rmsnorm(x[row:row + 1], w.final_norm, cfg.rms_norm_eps)
            logits = ref.linear(xl, w.lm_head)[0].float()
            tok[0] = int(torch.argmax(logits))
        if self.world > 1:
            dist.broadcast(tok, src=st.owner_of_last, group=self.group)
            dist.broadcast(logits, src=st.owner_of_last, group=self.group)
        return tok, (logits if return_logits else None)

    # ------------------------------------------------------------------ decode
    def _decode_meta(self, req_ids: Sequence[int]):
        """Per-step host metadata: positions, KV owner/slot per (row, layer), local KV lengths."""
        B = len(req_ids)
        pos = np.zeros(B, dtype=np.int32)
        owner = np.zeros((B, self.L), dtype=np.int32)
        slot = np.zeros((B, self.L), dtype=np.int32)
        ntok = np.zeros((self.L, B), dtype=np.int32)
        for b, rid in enumerate(req_ids):
            st = self.reqs[rid]
            t = st.decode_offset
            if t >= st.horizon:
                raise CapacityError(f"request {rid} exhausted its decode horizon {st.horizon}")
            pos[b] = st.context_len
            own = (st.assignee[t] == self.rank)
            if self.cuda:
                counts = st.kv.layer_counts
                full = np.nonzero(own & (counts + 1 > st.kv.capacity))[0]
                if full.size:
                    st.kv.check_room(int(full[0]))   # raises for the first full layer
                owner[b] = own
                slot[b] = counts
                ntok[:, b] = counts + own
            else:
                # legacy route: every rank keeps every decoded row
                owner[b] = 1 if self.legacy_decode else own
        return pos, owner, slot, ntok

    def _advance(self, req_ids: Sequence[int], owner: np.ndarray, pos: np.ndarray) -> None:
        for b, rid in enumerate(req_ids):
            st = self.reqs[rid]
            if self.cuda:
                li = np.nonzero(owner[b])[0]
                st.kv.slot_pos[li, st.kv.layer_counts[li]] = pos[b]
                st.kv.layer_counts += owner[b]
            st.decode_offset += 1
            st.context_len += 1

    @torch.no_grad()
    def decode_step(self, req_ids: Sequence[int], tokens: torch.Tensor,
                    logits: bool = True) -> torch.Tensor:
        """One greedy decode step for a batch of requests. `tokens` [B] holds each row's last
        token (int64 or int32, on the engine device). Returns the next tokens [B] (int64).
        `logits=False` promises that `last_logits` is not read for this step: on several ranks
        each one then runs the LM head over its own slice of the vocabulary only (the same
        tokens, bit for bit)."""
        B = len(req_ids)
        if B == 0:
            return tokens
        pos, owner, slot, ntok = self._decode_meta(req_ids)
        timing = self.perf.enabled
        if timing:
            t0 = time.perf_counter()
            if self.cuda:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
        if self.cuda:
            out = self._decode_cuda(req_ids, tokens, pos, owner, slot, ntok,
                                    split=self.split_head and not logits)
        else:
            out = self._decode_host(req_ids, tokens, pos, owner)
        if timing:
            if self.cuda:
                ev[1].record()
                ev[1].synchronize()
                ms = ev[0].elapsed_time(ev[1])
            else:
                ms = (time.perf_counter() - t0) * 1e3
            self._emit_decode(req_ids, tokens, pos, owner, ms)
        self._advance(req_ids, owner, pos)
        return out

    def _emit_decode(self, req_ids, tokens, pos, owner, ms: float) -> None:
        """`stationary_decode` perf event per row (the reference's schema,
        worker_sdk/tch_backend.rs:859-880). On the (O, LSE) exchange route every layer stores
        this rank's partial, H x (D + 1) float32 per row, into each other rank's slot: one hop,
        not N - 1. The whole batch step is one device-timed interval."""
        peers = self.world - 1
        part = self.H * (self.D + 1) * 4
        toks = tokens.view(-1).tolist()
        for b, rid in enumerate(req_ids):
            st = self.reqs[rid]
            n_msg = self.L * peers
            sent = recv = n_msg * part
            if self.legacy_decode:
                # this rank's partition rows (float32 K and V) go to every peer, every layer;
                # what arrives depends on the peers' partitions
                rows = sum(int(kv[3].sum()) for kv in st.host_kv)
                sent, recv = rows * 2 * self.Hkv * self.D * 4 * peers, -1
            self.perf.emit("stationary_decode", domain=self.rank, request_id=int(rid),
                           token=int(toks[b]), position=int(pos[b]), layers=self.L,
                           domains=self.world, token_offset=int(st.decode_offset),
                           decode_horizon=int(st.horizon), sends=n_msg, recvs=n_msg,
                           wire_sent_bytes=sent, wire_recv_bytes=recv,
                           hops_per_layer=1 if peers else 0,
                           kv_rows_appended=int(np.sum(owner[b])), batch=len(req_ids),
                           route="legacy_kv_resend" if self.legacy_decode else "o_lse_exchange",
                           recv_wait_ms=0.0, process_ms=ms, send_ms=0.0, total_ms=ms)

    def _graph_for(self, B: int) -> "DecodeGraph":
        g = self._graphs.get(B)
        if g is None:
            g = DecodeGraph(self, B)
            self._graphs[B] = g
        return g

    def _decode_cuda(self, req_ids, tokens, pos, owner, slot, ntok, split: bool = False):
        B = len(req_ids)
        bucket = 1 if B == 1 else 2 if B == 2 else 4 if B <= 4 else 8
        if B > self.max_batch or bucket > self.max_batch:
            raise CapacityError(f"decode batch {B} exceeds max_batch {self.max_batch}")
        g = self._graph_for(bucket)
        self._last_bucket = bucket
        self._last_split = split
        return g.run(req_ids, tokens, pos, owner, slot, ntok, split)

    def _decode_host(self, req_ids, tokens, pos, owner):
        w, cfg = self.w, self.cfg
        B = len(req_ids)
        x = w.embed[tokens.long().view(-1)].float()
        posn = torch.from_numpy(pos.astype(np.int64))
        for li, lw in enumerate(w.layers):
            h = ref.rmsnorm(x, lw.in_norm, cfg.rms_norm_eps)
            qkv = ref.linear(h, lw.wqkv, lw.bqkv)
            q = ref.apply_rope(qkv[:, : self.H * self.D].view(B, self.H, self.D), posn, cfg.rope_theta, cfg.rope_scaling)
            k = ref.apply_rope(qkv[:, self.H * self.D:(self.H + self.Hkv) * self.D].view(B, self.Hkv, self.D),
                               posn, cfg.rope_theta, cfg.rope_scaling)
            v = qkv[:, (self.H + self.Hkv) * self.D:].reshape(B, self.Hkv, self.D)
            outs = []
            for b, rid in enumerate(req_ids):
                st = self.reqs[rid]
                kv = st.host_kv[li]
                if owner[b, li]:
                    kv[0] = torch.cat([kv[0], k[b:b + 1]])
                    kv[1] = torch.cat([kv[1], v[b:b + 1]])
                    kv[2] = torch.cat([kv[2], posn[b:b + 1]])
                    kv[3] = torch.cat([kv[3], torch.tensor([not self.legacy_decode])])
                if self.legacy_decode:
                    # re-send every rank's partition rows (ring.rs:982-997), attend over them
                    # plus the replicated decoded rows; every rank gets the whole answer
                    sh = kv[3]
                    kk = torch.cat(self._gather_rows(kv[0][sh]) + [kv[0][~sh]])
                    vv = torch.cat(self._gather_rows(kv[1][sh]) + [kv[1][~sh]])
                    o, _ = ref.full_attention(q[b:b + 1], kk, vv, causal=False)
                    outs.append(o)
                    continue
                if kv[0].shape[0]:
                    o, lse = ref.full_attention(q[b:b + 1], kv[0], kv[1], causal=False)
                else:
                    o = torch.zeros(1, self.H, self.D)
                    lse = torch.full((self.H, 1), float("-inf"))
                os_ = self._gather_rows(o)
                ls_ = self._gather_rows(lse.transpose(0, 1).contiguous())
                om, _ = ref.merge_partials(os_, [l.transpose(0, 1) for l in ls_])
                outs.append(om)
            o = torch.cat(outs)
            x = x + ref.linear(o.reshape(B, self.H * self.D), lw.wo)
            h = ref.rmsnorm(x, lw.post_norm, cfg.rms_norm_eps)
            x = x + ref.linear(K.swiglu_from_interleaved(ref.linear(h, lw.wgu)), lw.wd)
        xl = ref.rmsnorm(x, w.final_norm, cfg.rms_norm_eps)
        logits = ref.linear(xl, w.lm_head)
        self._host_logits = logits
        return torch.argmax(logits, dim=-1)

    def last_logits(self, n: int) -> Optional[torch.Tensor]:
        """Logits [n, vocab] of the most recent decode step (for non-greedy sampling); None
        after a step run with `logits=False` on several ranks (no rank holds them all)."""
        if self.cuda:
            if not self._graphs or self._last_split:
                return None
            g = self._graphs.get(self._last_bucket)
            return None if g is None else g.logits[:n]
        return getattr(self, "_host_logits", None)

    # ------------------------------------------------------------------ continuation (sessions)
    def _segment_chunks(self, S: int, tickets: Sequence[int]) -> List[int]:
        from ..parallel.capacity import continuation_split
        return continuation_split(S, tickets)

    @torch.no_grad()
    def append(self, req_id: int, tokens: torch.Tensor, position_ids: Sequence[int],
               tickets: Sequence[int], return_logits: bool = False, extra_horizon: int = 128):
        """Continuation segment on a kept session: the segment's KV is placed capacity-weighted
        (vanilla split of the segment by `tickets`), existing KV never moves, and the segment's
        queries attend to the whole session through the ring. Returns (next_token, logits)."""
        st = self.reqs.get(req_id)
        if st is None:
            raise CapacityError(f"request {req_id} has no session KV on rank {self.rank}")
        S = int(tokens.numel())
        L0 = st.context_len
        if list(position_ids) != list(range(L0, L0 + S)):
            raise RingError(f"continuation positions must continue the session at {L0}")
        if L0 + S > self.max_context:
            raise CapacityError(f"session length {L0 + S} exceeds context capacity {self.max_context}")
        seg = self._segment_chunks(S, tickets)
        off = sum(seg[: self.rank])
        T = seg[self.rank]
        my_pos = np.arange(L0 + off, L0 + off + T, dtype=np.int64)
        last_owner = max(r for r in range(self.world) if seg[r] > 0)
        new_horizon = st.decode_offset + extra_horizon
        sched_tab = self._schedule(req_id, tickets, new_horizon, st.decode_offset, L0 + S)
        if self.cuda:
            kv = st.kv
            growth = int((sched_tab[st.decode_offset:] == self.rank).sum(0).max()) if extra_horizon else 0
            self.kv.extend(req_id, T + growth)
            kv.pt_device = torch.tensor(kv.pages, dtype=torch.int32, device=self.device)
            tok, logits = self._append_cuda(st, tokens.to(self.device)[off:off + T].int(), my_pos,
                                            L0 + S, last_owner, return_logits)
            for li in range(self.L):
                c = int(kv.layer_counts[li])
                kv.slot_pos[li, c:c + T] = my_pos
            kv.layer_counts += T
        else:
            tok, logits = self._append_host(st, tokens[off:off + T], my_pos, L0 + S, last_owner,
                                            return_logits)
        st.context_len = L0 + S
        st.assignee = sched_tab
        st.horizon = new_horizon
        return tok, logits

    def _append_cuda(self, st, ids, my_pos, Ltot, last_owner, return_logits):
        w, dev = self.w, self.device
        T = ids.numel()
        pos = torch.from_numpy(my_pos.astype(np.int32)).to(dev)
        kv = st.kv
        x = K.embedding(ids, w.embed) if T else torch.empty(0, self.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        xn = torch.empty_like(x)
        q_buf = torch.empty(T, self.H, self.D, dtype=torch.bfloat16, device=dev)
        o_buf = torch.empty_like(q_buf)
        for li, lw in enumerate(w.layers):
            c = int(kv.layer_counts[li])
            existing = torch.from_numpy(kv.slot_pos[li, :c].astype(np.int32)).to(dev)
            self.prefill_epoch += 1
            if T:
                K.rmsnorm(x, lw.in_norm, self.cfg.rms_norm_eps, out=xn)
            # continuation segments use the serial ring (every rank calls, with or without rows)
            o = self.attn.forward(xn, lw, LayerCall(st, li, pos, Ltot, q_buf, o_buf, self.prefill_epoch,
                                                    slot_base=c, existing=existing))
            if T:
                K.gemm(o, lw.wo, "residual", residual=x)
                K.rmsnorm(x, lw.post_norm, self.cfg.rms_norm_eps, out=xn)
                g = K.gemm(xn, lw.wgu, "swiglu")
                K.gemm(g, lw.wd, "residual", residual=x)
        st_last = dataclasses.replace(st, positions=my_pos, prompt_len=Ltot, owner_of_last=last_owner)
        return self._first_token_cuda(st_last, x, return_logits)

    def _append_host(self, st, ids, my_pos, Ltot, last_owner, return_logits):
        w, cfg = self.w, self.cfg
        T = ids.numel()
        pos = positions_tensor(my_pos, self.device)
        x = w.embed[ids.long()].float()
        for li, lw in enumerate(w.layers):
            h = ref.rmsnorm(x, lw.in_norm, cfg.rms_norm_eps) if T else x
            # every rank takes part in the backend's gathers, with or without rows
            o = self.attn.forward(h, lw, LayerCall(st, li, pos, Ltot, existing=st.host_kv[li][2]))
            if T:
                x = x + ref.linear(o, lw.wo)
                h = ref.rmsnorm(x, lw.post_norm, cfg.rms_norm_eps)
                x = x + ref.linear(K.swiglu_from_interleaved(ref.linear(h, lw.wgu)), lw.wd)
        tok = torch.zeros(1, dtype=torch.int64)
        logits = torch.zeros(cfg.vocab_size, dtype=torch.float32)
        if self.rank == last_owner:
            xl = ref.rmsnorm(x[-1:], w.final_norm, cfg.rms_norm_eps)
            logits = ref.linear(xl, w.lm_head)[0].float()
            tok[0] = int(torch.argmax(logits))
        if self.world > 1:
            dist.broadcast(tok, src=last_owner, group=self.group)
            dist.broadcast(logits, src=last_owner, group=self.group)
        return tok, (logits if return_logits else None)

    # ------------------------------------------------------------------ release / generate
    def release(self, req_id: int) -> bool:
        st = self.reqs.pop(req_id, None)
        if st is None:
            return False
        if self.cuda:
            self.kv.release(req_id)
        return True

    @torch.no_grad()
    def generate(self, req_id: int, prompt_ids: torch.Tensor, max_new_tokens: int,
                 chunks: Sequence[int], strategy=None, tickets=None,
                 stop_ids: Optional[Sequence[int]] = None) -> torch.Tensor:
        """Greedy generation (SPMD across ranks). Returns the generated ids [n] on the device.

        The decode loop never reads tokens back to the host unless `stop_ids` is given."""
        first, _ = self.prefill(req_id, prompt_ids, chunks, strategy, decode_horizon=max(1, max_new_tokens),
                                tickets=tickets)
        toks = [first.view(1)]
        cur = first.view(1)
        try:
            for _ in range(max_new_tokens - 1):
                cur = self.decode_step([req_id], cur, logits=False).view(1)
                toks.append(cur)
                if stop_ids is not None and int(cur) in stop_ids:
                    break
        finally:
            self.release(req_id)
        return torch.cat(toks)

    @torch.no_grad()
    def warmup(self, batch_sizes: Optional[Sequence[int]] = None) -> None:
        """Run short dummy requests through every decode batch bucket (1, 2, 4, 8 up to
        max_batch) so kernel set-up and the decode CUDA-graph captures happen before the first
        real request instead of inside its latency. SPMD: every rank calls it at the same point.
        The dummy request ids (from 2^40) never meet a coordinator's ids."""
        sizes = batch_sizes or [b for b in (1, 2, 4, 8) if b <= self.max_batch]
        prompt = torch.arange(max(8, self.world), dtype=torch.int64) % self.cfg.vocab_size
        for b in sizes:
            self.generate_batch([prompt] * b, 2, first_id=(1 << 40) + 16 * b)
            if self.cuda and self.split_head:   # the logits-keeping graph (sampled requests)
                self.generate_batch([prompt] * b, 2, first_id=(1 << 40) + 16 * b + 8, logits=True)

    def generate_batch(self, prompts: Sequence[torch.Tensor], max_new_tokens: int,
                       chunks_for=None, strategy=None, first_id: int = 1 << 20,
                       logits: bool = False) -> List[torch.Tensor]:
        """Greedy generation for several prompts (rust/src/model/generator.rs:123-270
        `BatchGenerator`): each prompt is prefilled (with its own chunk split), then every decode
        step advances all rows in one batched step. Returns the generated ids per prompt.
        `logits=True` keeps every step's logits (the whole LM head on every rank)."""
        from ..parallel.capacity import equal_chunks
        chunks_for = chunks_for or (lambda n: equal_chunks(n, self.world))
        rids = list(range(first_id, first_id + len(prompts)))
        firsts = []
        try:
            for rid, p in zip(rids, prompts):
                tok, _ = self.prefill(rid, p, chunks_for(int(p.numel())), strategy,
                                      decode_horizon=max(1, max_new_tokens))
                firsts.append(tok.view(1))
            cur = torch.cat(firsts)
            outs = [cur]
            for _ in range(max_new_tokens - 1):
                cur = self.decode_step(rids, cur, logits=logits).view(-1)
                outs.append(cur)
        finally:
            for rid in rids:
                self.release(rid)
        allt = torch.stack(outs, dim=1)
        return [allt[i] for i in range(len(prompts))]


class DecodeGraph:
    """Static buffers + a captured CUDA graph for one decode batch size."""

    def __init__(self, eng: LlamaCPEngine, B: int):
        self.e = eng
        self.B = B
        dev = eng.device
        cfg = eng.cfg
        L = eng.L
        self.max_pages = eng.kv.alloc.num_pages
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.out_tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.owner = torch.zeros(B, L, dtype=torch.int32, device=dev)
        self.slot = torch.zeros(B, L, dtype=torch.int32, device=dev)
        self.ntok = torch.zeros(L, B, dtype=torch.int32, device=dev)
        self.pt = torch.zeros(B, self.max_pages, dtype=torch.int32, device=dev)
        pin = dict(pin_memory=True)
        self.h_pos = torch.zeros(B, dtype=torch.int32, **pin)
        self.h_owner = torch.zeros(B, L, dtype=torch.int32, **pin)
        self.h_slot = torch.zeros(B, L, dtype=torch.int32, **pin)
        self.h_ntok = torch.zeros(L, B, dtype=torch.int32, **pin)
        self.h_pt = torch.zeros(B, self.max_pages, dtype=torch.int32, **pin)
        self.x = torch.zeros(B, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        self.xn = torch.zeros_like(self.x)
        self.q = torch.zeros(B, eng.H, eng.D, dtype=torch.bfloat16, device=dev)
        self.o = torch.zeros(B, eng.H * eng.D, dtype=torch.bfloat16, device=dev)
        self.g = torch.zeros(B, eng.w.intermediate_padded, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
        self.am = torch.zeros(B, dtype=torch.int64, device=dev)
        # one wave: resident decode-attention CTAs per SM x SMs, spread over the (row, KV head) pairs
        occ = max(1, int(native().decode_attn_ctas_per_sm(eng.D, eng.H // eng.Hkv)))
        self.splits = max(1, min(128, (occ * eng.num_sms) // (B * eng.Hkv)))  # floor: never a 2nd wave
        if eng.env.decode_splits > 0:
            self.splits = min(self.splits, eng.env.decode_splits)
        self.part_o = torch.zeros(B * eng.H * self.splits * eng.D, dtype=torch.float32, device=dev)
        self.part_l = torch.zeros(B * eng.H * self.splits, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(B * eng.Hkv + 1, dtype=torch.int32, device=dev)
        # one zeroed barrier-counter pair per GEMV chain launch site (one per layer)
        self.chain_ctr = torch.zeros(L, 2, dtype=torch.int32, device=dev)
        self.graphs: Dict[bool, torch.cuda.CUDAGraph] = {}
        self.graph_launches: Dict[bool, int] = {}
        self.copied = None

    def body(self, split: bool = False) -> None:
        e, w, cfg = self.e, self.e.w, self.e.cfg
        rt = e.rt
        nat = native()
        nat.add_u64(e.dec_step, 1)
        launches.count()
        K.embedding(self.tokens, w.embed, out=self.x)
        nat.fill_u64(self.am, 0)
        launches.count()
        eps = cfg.rms_norm_eps
        single = e.world == 1
        head = e.lm_head_slice if split else w.lm_head
        pf = self.prefetch_plan(head)
        L = len(w.layers)
        # HCP_DECODE_CHAIN=1: the GEMVs between two attentions (output projection, gate/up,
        # down, then the next layer's QKV projection or the LM head) run as one cooperative
        # chain launch with grid barriers between them (batches of up to 4 rows; measured
        # slower than the four launches, so off by default)
        chain = e.env.decode_chain and self.B <= 4

        def qkv(li: int) -> None:
            lw = w.layers[li]
            # RMSNorm + QKV GEMV whose epilogue applies RoPE, writes q and appends k/v on the owner
            rt.qkv_gemv_rope(self.x, lw.wqkv, lw.bqkv, lw.in_norm, eps, self.pos, e.cos, e.sin, li,
                             self.pt, self.owner, self.slot, self.q, prefetch=pf[li][0])

        def lm_head() -> None:
            if split:
                # greedy step, head split over the vocabulary: this rank's rows only (no logits),
                # then every rank stores its packed maxima into every rank's slots and takes the
                # max
                K.gemv(self.x, e.lm_head_slice, "argmax", argmax=self.am, norm_w=w.final_norm,
                       eps=eps, index_base=e.vocab_lo)
            else:
                K.gemv(self.x, w.lm_head, "argmax", y_f32=self.logits, argmax=self.am,
                       norm_w=w.final_norm, eps=eps)

        head_done = False
        for li, lw in enumerate(w.layers):
            if li == 0 or not chain:       # else the previous layer's chain ran it
                qkv(li)
            # split-KV attention; on one rank its last CTA writes the layer output directly.
            # With several ranks the rank's (O, LSE) partial goes into every rank's slots and
            # the log-sum-exp combine in rank order follows a bounded wait for the other ranks'
            # partials: in a launch of its own (HCP_DECODE_COMBINE=launch, the default and the
            # fastest measured), in the output projection's prologue (=gemv: every CTA of the
            # GEMV waits and combines the same partials) or in the attention kernel's last CTA
            # of each (row, KV head) (=attn)
            mode = "single" if single else e.env.decode_combine
            rt.decode_attn(self.q, li, self.pt, self.ntok[li], e.scale, self.splits, self.part_o,
                           self.part_l, self.counters, e.dec_step, e.L, li + 1,
                           self.o if single else None, self.o if mode == "attn" else None,
                           prefetch=pf[li][1])
            if mode == "launch":
                rt.decode_combine(self.o, self.B, e.H, e.dec_step, e.L, li + 1)
            launches.count((3 if mode == "launch" else 2) - (1 if chain and li > 0 else 0))
            if chain:
                nat.gemv_chain_begin()
            if mode == "gemv":
                rt.o_proj_combine(self.o, lw.wo, self.x, e.dec_step, e.L, li + 1)
                launches.count()
            else:
                K.gemv(self.o, lw.wo, "residual", y_bf16=self.x, prefetch=pf[li][2])
            K.gemv(self.x, lw.wgu, "swiglu", y_bf16=self.g, norm_w=lw.post_norm, eps=eps,
                   prefetch=pf[li][3])
            K.gemv(self.g, lw.wd, "residual", y_bf16=self.x)
            if chain:
                last = li + 1 == L
                if last:
                    lm_head()
                    head_done = True
                else:
                    qkv(li + 1)
                ran = nat.gemv_chain_end(self.chain_ctr[li])
                # counted so far in the chain: o, gate/up, down (+ the LM head); launched: one
                # chain kernel, or the four GEMVs one by one
                launches.count((1 if ran else 4) - (4 if last else 3))
        if not head_done:
            lm_head()
        if split:
            rt.argmax_exchange(self.am, e.dec_step, self.tokens, self.out_tok)
        else:
            nat.argmax_finalize(self.am, self.tokens, self.out_tok)
        launches.count()

    def prefetch_plan(self, head: torch.Tensor) -> list:
        """Per layer, the weights each decode kernel pulls into L2 for a later kernel while it
        runs (HCP_DECODE_PREFETCH=1 or 2; 3 keeps only the first and the last): the QKV GEMV
        the output projection's, the attention (which streams KV at a fraction of HBM
        bandwidth) the gate/up weights, the output projection the down projection's, gate/up
        the next layer's QKV weights or, after the last layer, an LM head of at most 96 MB (the
        vocabulary slice on several ranks)."""
        w = self.e.w
        L = len(w.layers)
        mode = self.e.env.decode_prefetch
        if not mode:
            return [([], [], [], [])] * L
        plan = []
        for li, lw in enumerate(w.layers):
            if li + 1 < L:
                nxt = [w.layers[li + 1].wqkv]
            else:
                nxt = [head] if head.numel() * head.element_size() <= (96 << 20) else []
            if mode == 3:   # only the small projections' weights
                plan.append(([lw.wo], [], [], nxt if li + 1 < L else []))
            else:
                plan.append(([lw.wo], [lw.wgu], [lw.wd], nxt))
        return plan

    def run(self, req_ids, tokens, pos, owner, slot, ntok, split: bool = False) -> torch.Tensor:
        n = len(req_ids)
        # the pinned host buffers are reused every step: wait until the previous step's
        # host-to-device copies have executed before overwriting them
        if self.copied is not None:
            self.copied.synchronize()
        self.h_pos.zero_()
        self.h_owner.zero_()
        self.h_slot.zero_()
        self.h_ntok.zero_()
        self.h_pos[:n] = torch.from_numpy(pos)
        self.h_owner[:n] = torch.from_numpy(owner)
        self.h_slot[:n] = torch.from_numpy(slot)
        self.h_ntok[:, :n] = torch.from_numpy(ntok)
        for b, rid in enumerate(req_ids):
            pages = self.e.reqs[rid].kv.pages
            self.h_pt[b, : len(pages)] = torch.tensor(pages, dtype=torch.int32)
        self.pos.copy_(self.h_pos, non_blocking=True)
        self.owner.copy_(self.h_owner, non_blocking=True)
        self.slot.copy_(self.h_slot, non_blocking=True)
        self.ntok.copy_(self.h_ntok, non_blocking=True)
        self.pt.copy_(self.h_pt, non_blocking=True)
        if self.copied is None:
            self.copied = torch.cuda.Event()
        self.copied.record()
        if n < self.B:
            self.tokens.zero_()
        self.tokens[:n].copy_(tokens.view(-1)[:n].to(torch.int32))
        if not self.e.use_graphs:
            self.body(split)
        else:
            graph = self.graphs.get(split)
            if graph is None:
                # every kernel of the body writes into preallocated buffers (function attributes
                # and TMA descriptors are host-side calls, legal during capture), so the graph is
                # captured directly (no eager warm-up step, which would advance the cross-rank
                # exchange epochs and overwrite `tokens`). One graph per LM-head mode; both
                # share the buffers.
                graph = torch.cuda.CUDAGraph()
                with launches.capture() as cap:
                    with torch.cuda.graph(graph):
                        self.body(split)
                self.graphs[split] = graph
                self.graph_launches[split] = cap.launches
            if self.e.env.nvtx:
                torch.cuda.nvtx.range_push(f"decode step B={self.B}")
            graph.replay()
            if self.e.env.nvtx:
                torch.cuda.nvtx.range_pop()
            launches.count(self.graph_launches[split])
        return self.out_tok[:n].clone()
