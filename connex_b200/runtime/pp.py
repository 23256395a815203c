"""Elastic pipeline-parallel serving of the Llama decoder on sm_100a.

A pipeline stage owns layers ``[l0, l1)`` of the model (their weights and
their paged KV cache); stage 0 also owns the embedding, the last stage the
final norm, LM head and the greedy sampler.  Between stages only the
residual stream ``x`` ([tokens, hidden] bf16) travels, over the endpoint's
data plane (elastic NCCL pair links inside a box).

:class:`StageRuntime` is a stage's compute for the step protocol: a step
carries ``request_ids``, ``cx_ctx`` (tokens of each request already in the
KV cache before this step) and ``n_new`` (tokens of each request in this
step: the prompt for a prefill, 1 for a decode).  A stage allocates KV
blocks per request on demand and answers ``kv_held`` for the handover rules,
so after a failover the rows whose KV is not here come back as
``cx_missing`` and stage 0 prefills them again (reference semantics:
``connex/pp/handover.py``, ``connex/pp/link.py``).

Weights are random N(0, 0.02) per layer from ``seed + layer`` so a split
model equals the unsplit one layer for layer (tests compare them).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from connex.pp.handover import CX_CTX, REQUEST_IDS
from connex_b200 import ops
from connex_b200.models.llama import LayerWeights, LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache


def layer_weights(cfg: LlamaConfig, layer: int, device, seed: int = 0, std: float = 0.02) -> LayerWeights:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + layer + 1)

    def rnd(*shape):
        t = torch.empty(*shape, dtype=torch.bfloat16, device=device)
        t.normal_(0.0, std, generator=g)
        return t
    ones = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device)
    gate, up = rnd(cfg.ffn, cfg.hidden), rnd(cfg.ffn, cfg.hidden)
    return LayerWeights(attn_norm=ones, wqkv=rnd(cfg.qkv_dim, cfg.hidden), wo=rnd(cfg.hidden, cfg.heads * cfg.head_dim),
                        mlp_norm=ones.clone(), w13=ops.interleave_gate_up(gate, up), w2=rnd(cfg.hidden, cfg.ffn))


def stage_weights(cfg: LlamaConfig, l0: int, l1: int, device, seed: int = 0, std: float = 0.02) -> LlamaWeights:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + 999)

    def rnd(*shape):
        t = torch.empty(*shape, dtype=torch.bfloat16, device=device)
        t.normal_(0.0, std, generator=g)
        return t
    embed = rnd(cfg.vocab_size, cfg.hidden)            # same draw order on every stage
    head = rnd(cfg.vocab_size, cfg.hidden)
    return LlamaWeights(cfg=cfg, embed=embed if l0 == 0 else None,
                        layers=[layer_weights(cfg, l, device, seed, std) for l in range(l0, l1)],
                        final_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device) if l1 == cfg.layers
                        else None, lm_head=head if l1 == cfg.layers else None)


class StageModel(LlamaModel):
    """Layers ``[l0, l1)`` of the decoder on their own KV cache."""

    def __init__(self, weights: LlamaWeights, l0: int, l1: int, cache: PagedKVCache, max_tokens: int,
                 max_batch: int = 256, device=None, tp=None):
        self.l0, self.l1 = l0, l1
        self.is_first, self.is_last = l0 == 0, l1 == weights.cfg.layers
        dev = torch.device(device) if device is not None else weights.layers[0].wqkv.device
        if weights.embed is None:          # LlamaModel reads the device from the embedding
            weights.embed = torch.empty(0, weights.cfg.hidden, dtype=torch.bfloat16, device=dev)
        super().__init__(weights, cache, max_tokens, max_batch, tp=tp)

    def _next_norm(self, i: int):
        if i + 1 < len(self.w.layers):
            return self.w.layers[i + 1].attn_norm
        return self.w.final_norm if self.is_last else None

    def _tail(self, i: int, T: int) -> None:
        cfg, lw = self.cfg, self.w.layers[i]
        x, h = self.x[:T], self.h[:T]
        self._residual_gemm(self.attn[:T], lw.wo, x)
        ops.rmsnorm(x, lw.mlp_norm, cfg.eps, out=h)
        ops.gemm(h, lw.w13, self.mid[:T], silu_mul=True, status=self.status)
        self._residual_gemm(self.mid[:T], lw.w2, x)
        nw = self._next_norm(i)
        if nw is not None:
            ops.rmsnorm(x, nw, self.cfg.eps, out=h)

    def _enter(self, inp: torch.Tensor, T: int) -> None:
        if self.is_first:
            ops.embedding(inp, self.w.embed, self.x[:T], status=self.status)
        else:
            self.x[:T].copy_(inp)
        ops.rmsnorm(self.x[:T], self.w.layers[0].attn_norm, self.cfg.eps, out=self.h[:T])

    def run(self, inp: torch.Tensor, positions, slots, *, prefill: bool, tile_info=None, block_tables=None,
            ctx_lens=None, max_ctx: int = 0, workspace=None, rows=None, B: int = 0, n_dec: Optional[int] = None):
        """Ids (first stage) or the residual stream in; the residual stream
        (``x[:T]``) or, on the last stage, the greedy next ids of ``rows`` out.

        ``n_dec`` set: a mixed step -- the first ``n_dec`` rows are decode
        rows (paged decode attention over ``block_tables[:n_dec]`` /
        ``ctx_lens``), the rest are prefill chunks that continue cached
        sequences (the paged prefill kernel over ``block_tables[n_dec:]`` and
        ``tile_info`` of width 5); every GEMM runs once over all rows."""
        cfg, T = self.cfg, inp.shape[0]
        assert T <= self.max_tokens
        self._enter(inp, T)
        for i, lw in enumerate(self.w.layers):
            qkv = self.qkv[:T]
            ops.gemm(self.h[:T], lw.wqkv, qkv, status=self.status)
            ops.rope_cache(qkv, positions, self.cos_sin, cfg.heads, cfg.kv_heads, slots, self.cache.k(i),
                           self.cache.v(i), status=self.status)
            if n_dec is not None:
                if n_dec:
                    ops.decode_attention(qkv[:n_dec], self.cache.k(i), self.cache.v(i), block_tables[:n_dec],
                                         ctx_lens, cfg.heads, max_ctx, workspace, out=self.attn[:n_dec])
                if T > n_dec:
                    ops.prefill_attention_paged(qkv[n_dec:], self.cache.k(i), self.cache.v(i), block_tables[n_dec:],
                                                tile_info, cfg.heads, cfg.kv_heads, out=self.attn[n_dec:T],
                                                status=self.status)
            elif prefill:
                ops.prefill_attention(qkv, tile_info, cfg.heads, cfg.kv_heads, out=self.attn[:T])
            else:
                ops.decode_attention(qkv, self.cache.k(i), self.cache.v(i), block_tables, ctx_lens, cfg.heads,
                                     max_ctx, workspace, out=self.attn[:T])
            self._tail(i, T)
        if self.is_last:
            return self._head(rows, B)
        return self.x[:T]


class StageRuntime:
    """One stage's compute for the step protocol (``StageWorker`` compute + hooks)."""

    def __init__(self, cfg: LlamaConfig, l0: int, l1: int, device, num_blocks: int, max_tokens: int,
                 max_batch: int = 256, max_ctx: int = 8192, seed: int = 0, weights: Optional[LlamaWeights] = None,
                 tp=None):
        """``weights``: layers ``[l0, l1)`` already on ``device`` (e.g. from
        :func:`connex_b200.models.hf.load_llama`); random from ``seed`` if absent."""
        self.cfg = cfg
        self.device = torch.device(device)
        if weights is not None and len(weights.layers) != l1 - l0:
            raise ValueError(f"weights hold {len(weights.layers)} layers, the stage owns {l1 - l0}")
        self.weights = weights if weights is not None else stage_weights(cfg, l0, l1, self.device, seed)
        stage_cfg = LlamaConfig(**{**cfg.__dict__, "layers": l1 - l0})
        self.cache = PagedKVCache(stage_cfg, num_blocks, self.device)
        self.model = StageModel(self.weights, l0, l1, self.cache, max_tokens, max_batch, self.device, tp=tp)
        self.model.cfg = cfg
        self.bs = cfg.block_size
        self.max_ctx = max_ctx
        self.tables: Dict[object, List[int]] = {}
        self.held: Dict[object, int] = {}
        self.ws = ops.decode_workspace(max_batch, cfg.heads, max_ctx, self.device)
        self.steps = 0
        self.act: Optional[torch.Tensor] = None      # activation log (non-last stages)
        self.act_slot: Dict[object, int] = {}
        self.graphs: Optional[Dict[int, tuple]] = None

    # ------------------------------------------------------------ CUDA graphs
    def enable_decode_graphs(self, buckets: Optional[Sequence[int]] = None) -> None:
        """Replay the decode step from CUDA graphs, one per batch bucket
        (captured on first use): ~10 launches per layer become one graph
        launch, which is what bounds a small-batch decode step.

        The graphs read static device buffers (ids or the residual stream,
        positions, slots, context lengths, block tables over ``max_ctx``);
        each step stages them in one pinned host buffer and copies it up.
        Rows between the batch and its bucket point at a reserved trash KV
        block, so padding never writes a live request's cache.  The split-K
        workspace is sized for the largest bucket before any capture, so no
        captured pointer is ever reallocated."""
        if self.device.type != "cuda":
            return
        mb = self.model.max_batch
        bk = sorted({b for b in (buckets or (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)) if b <= mb} | {mb})
        self.g_buckets = bk
        top = bk[-1]
        self.g_mb = -(-self.max_ctx // self.bs)
        n_i32 = 3 * top + top * self.g_mb
        self.g_i32 = torch.zeros(n_i32, dtype=torch.int32, device=self.device)
        self.g_slots = torch.zeros(top, dtype=torch.int64, device=self.device)
        self.g_rows = torch.arange(top, dtype=torch.int32, device=self.device)
        self.g_x = None if self.model.is_first else torch.zeros(top, self.cfg.hidden, dtype=torch.bfloat16,
                                                                  device=self.device)
        self.h_i32 = torch.zeros(n_i32, dtype=torch.int32).pin_memory()
        self.h_slots = torch.zeros(top, dtype=torch.int64).pin_memory()
        self.h_done = torch.cuda.Event()
        self.trash = self.cache.allocate(1)[0]
        widths = [lw.wqkv.shape[0] for lw in self.weights.layers] + [self.cfg.hidden, 2 * self.cfg.ffn]
        if self.model.is_last:
            widths.append(self.weights.lm_head.shape[0])
        ops._split_workspace(self.device, top * max(widths))
        self.graphs = {}

    def _g_views(self, Bb: int):
        top, MB = self.g_buckets[-1], self.g_mb
        i = self.g_i32
        return (i[0:Bb], i[top:top + Bb], i[2 * top:2 * top + Bb], i[3 * top:].view(top, MB)[:Bb],
                self.g_slots[:Bb], self.g_rows[:Bb])

    def _g_body(self, Bb: int) -> torch.Tensor:
        ids, pos, lens, bt, slots, rows = self._g_views(Bb)
        inp = ids if self.model.is_first else self.g_x[:Bb]
        return self.model.run(inp, pos, slots, prefill=False, block_tables=bt, ctx_lens=lens, max_ctx=self.max_ctx,
                              workspace=self.ws, rows=rows, B=Bb)

    def _g_fill(self, B: int, Bb: int, pos, slots, lens, tables) -> None:
        """Stage one step's metadata; rows [B, Bb) read and write only the trash block."""
        top, MB = self.g_buckets[-1], self.g_mb
        self.h_done.synchronize()            # the previous step's upload has left this buffer
        h = self.h_i32
        h[top:top + Bb] = 0
        h[top:top + B] = torch.tensor(pos, dtype=torch.int32)
        h[2 * top:2 * top + Bb] = 1
        h[2 * top:2 * top + B] = torch.tensor(lens, dtype=torch.int32)
        bt = h[3 * top:].view(top, MB)
        bt[:Bb] = self.trash
        for i, t in enumerate(tables):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        self.h_slots[:Bb] = self.trash * self.bs
        self.h_slots[:B] = torch.tensor(slots, dtype=torch.int64)
        self.g_i32[top:].copy_(h[top:], non_blocking=True)
        self.g_slots[:Bb].copy_(self.h_slots[:Bb], non_blocking=True)
        self.h_done.record()

    def _g_decode(self, inp: torch.Tensor, B: int, pos, slots, lens, tables) -> torch.Tensor:
        Bb = next(b for b in self.g_buckets if b >= B)
        ids, *_ = self._g_views(Bb)
        if self.model.is_first:
            ids[:B].copy_(inp)
            if Bb > B:
                ids[B:].zero_()
        else:
            self.g_x[:B].copy_(inp)
        self._g_fill(B, Bb, pos, slots, lens, tables)
        if Bb not in self.graphs:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self._g_body(Bb)                 # warm-up outside the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self._g_body(Bb)
            self.graphs[Bb] = (g, out)
            self._g_fill(B, Bb, pos, slots, lens, tables)   # the warm-up ran on these buffers too
        g, out = self.graphs[Bb]
        g.replay()
        return out[:B]

    def enable_activation_log(self, max_requests: int) -> None:
        """Keep every output row of this stage per request ([requests, max_ctx,
        hidden] bf16, ~0.6 GB for 64 x 1280 x 4096).  After a failover the
        next stage's new replica is refilled by replaying these rows
        (:meth:`replay`) instead of recomputing this stage's layers."""
        if self.model.is_last:
            return
        self.act = torch.empty(max_requests, self.max_ctx, self.cfg.hidden, dtype=torch.bfloat16,
                               device=self.device)

    def _log(self, rids, ctx, n_new, out) -> None:
        slots, poss = [], []
        for r, c, n in zip(rids, ctx, n_new):
            sl = self.act_slot.get(r)
            if sl is None:
                sl = self.act_slot[r] = len(self.act_slot)
                if sl >= self.act.shape[0]:
                    raise MemoryError("activation log full")
            slots += [sl] * n
            poss += range(c, c + n)
        idx = (torch.tensor(slots, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True),
               torch.tensor(poss, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True))
        self.act.index_put_(idx, out)

    def replay(self, rids) -> tuple:
        """(rows [sum of tokens, hidden], tokens per request) of the logged
        outputs of ``rids`` -- the input of a re-prefill on the next stage."""
        lens = [self.held[r] for r in rids]
        x = torch.cat([self.act[self.act_slot[r], :n] for r, n in zip(rids, lens)])
        return x, lens

    # EngineHooks
    def kv_held(self, rid) -> int:
        return self.held.get(rid, 0)

    def release(self, rids) -> None:
        for r in rids:
            self.held.pop(r, None)
            self.cache.free(self.tables.pop(r, []))

    def reprefill(self, rids) -> None:
        pass

    def abort(self, rids) -> None:
        self.release(rids)

    def _blocks_for(self, rid, upto: int) -> List[int]:
        t = self.tables.setdefault(rid, [])
        need = -(-upto // self.bs)
        if len(t) < need:
            t += self.cache.allocate(need - len(t))
        return t

    def compute(self, td: dict, missing: Sequence) -> dict:
        if td.get("kind") == "warmup":      # link set-up step: echo, no model work
            return {"kind": "warmup", "w": td["w"].clone()}
        rids = list(td[REQUEST_IDS])
        ctx = list(td[CX_CTX])
        n_new = list(td["n_new"])
        kind = td["kind"]
        if kind == "prefill" and any(ctx):      # chunks that continue cached sequences
            kind = "mixed"
        n_dec = int(td.get("n_dec", 0)) if kind == "mixed" else None
        prefill = kind == "prefill"
        miss = set(missing)
        pos, slots, lens = [], [], []
        for r, c, n in zip(rids, ctx, n_new):
            if r in miss:
                self.release([r])
            t = self._blocks_for(r, c + n)
            for p in range(c, c + n):
                pos.append(p)
                slots.append(t[p // self.bs] * self.bs + p % self.bs)
            lens.append(c + n)
        dev = self.device
        B = len(rids)
        inp = td["ids"] if self.model.is_first else td["x"]
        graph = kind == "decode" and self.graphs is not None and B <= self.g_buckets[-1]
        if not graph:
            positions = torch.tensor(pos, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            slot_t = torch.tensor(slots, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
        kw = {}
        last_rows, start = [], 0
        for n in n_new:                 # each row's last token: its next id comes from there
            start += n
            last_rows.append(start - 1)
        if prefill:
            kw["tile_info"] = ops.prefill_tile_info(n_new, dev)
            kw["rows"] = torch.tensor(last_rows, dtype=torch.int32, device=dev)
        elif n_dec is not None:
            if any(n != 1 for n in n_new[:n_dec]):
                raise ValueError("a mixed step's decode rows carry one token each")
            mb = -(-max(lens) // self.bs)
            bt = torch.zeros(B, mb, dtype=torch.int32)
            for i, r in enumerate(rids):
                t = self.tables[r]
                bt[i, :len(t)] = torch.tensor(t[:mb], dtype=torch.int32)
            kw.update(n_dec=n_dec, block_tables=bt.pin_memory().to(dev, non_blocking=True),
                      tile_info=ops.prefill_tile_info(n_new[n_dec:], dev, ctx=ctx[n_dec:]),
                      rows=torch.tensor(last_rows, dtype=torch.int32).pin_memory().to(dev, non_blocking=True))
            if n_dec:
                kw.update(ctx_lens=torch.tensor(lens[:n_dec], dtype=torch.int32).pin_memory().to(dev, non_blocking=True),
                          max_ctx=max(lens[:n_dec]), workspace=self.ws)
        elif graph:
            out = self._g_decode(inp, B, pos, slots, lens, [self.tables[r] for r in rids])
            kw = None
        else:
            mb = -(-max(lens) // self.bs)
            bt = torch.zeros(B, mb, dtype=torch.int32)
            for i, r in enumerate(rids):
                t = self.tables[r]
                bt[i, :len(t)] = torch.tensor(t[:mb], dtype=torch.int32)
            kw.update(block_tables=bt.pin_memory().to(dev, non_blocking=True),
                      ctx_lens=torch.tensor(lens, dtype=torch.int32).pin_memory().to(dev, non_blocking=True),
                      max_ctx=max(lens), workspace=self.ws,
                      rows=torch.arange(B, dtype=torch.int32, device=dev))
        if kw is not None:
            out = self.model.run(inp, positions, slot_t, prefill=prefill, B=B, **kw)
        if self.act is not None:
            self._log(rids, ctx, n_new, out)
        for r, c, n in zip(rids, ctx, n_new):
            if r in miss:           # computed without its KV: not held here; stage 0 prefills it again
                self.release([r])
            else:
                self.held[r] = c + n
        self.steps += 1
        res = {"kind": td["kind"], "n_new": n_new}
        if n_dec is not None:
            res["n_dec"] = n_dec
        # a copy: the model's buffers are rewritten by the next step while the
        # link may still be sending this one
        res["next" if self.model.is_last else "x"] = out.clone()
        return res
