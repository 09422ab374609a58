"""Greedy decode over a paged KV cache, captured in a CUDA graph.

This replaces lightserve's static-buffer full-recompute decode
(``model/cuda_graph_decode.py:108-149``, which re-runs the whole causal
forward over ``[B, max_seq_len]`` every step) with an incremental decode: one
new token per sequence per step, its K/V written into a paged cache whose
block tables come from ``lightserve_b200.engine.BlockManager`` (lightserve's
``engine/block_manager.py`` API). The harness shape is the reference's:
side-stream warm-up before capture (``:129-135``), one captured step
(``:137-139``), replay per token, greedy ``argmax`` of the newest position's
logits (``:114-118``).

Per step and layer: fused add+RMSNorm (lsb kernel) -> fused QKV projection
-> ``rope_kv_write`` (lsb kernel: RoPE at each sequence's position, K/V into
the cache slot from the block table, context lengths) ->
``paged_decode_attention`` (lsb kernel) -> O projection -> add+RMSNorm ->
fused gate|up projection -> SwiGLU (lsb kernel) -> down projection; then the
final norm and the lm_head projection. The projections run on cuBLAS, or
with ``use_lsb_linear`` (bf16/fp16, at most 128 sequences) on
``lsb_linear`` (tcgen05 weight streaming). All buffers are static, so a step
is graph-capturable.

Prefill: with a bf16/fp16 model and head_dim 64 or 128, every admitted prompt
runs in ONE packed forward ([sum of prompt lengths, hidden]: the GEMMs see
all prompt tokens at once, ``rope_kv_write_slots`` rotates q/k and fills the
cache through each token's slot, ``flash_attention_varlen`` attends within
each prompt); other models prefill one request at a time through
``llama_forward``.

Block reservation: at admission the runner asks the block manager for every
block the request will need over ``max_new_tokens`` (``allocate`` for the
prompt, then the same ``append_slot`` sequence the scheduler would issue one
token at a time), so replays never need new host-side table entries.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..engine import BlockManager, Request
from ..kernels.fused_rmsnorm_residual import fused_add_rmsnorm
from ..kernels.fused_swiglu import silu_and_mul
from ..kernels.flash_attention import flash_attention_varlen
from ..kernels.linear import MAX_ROWS as LINEAR_MAX_ROWS
from ..kernels.linear import linear, pack_linear_weight
from ..kernels.sampling import greedy_next
from ..kernels.paged_attention import (paged_decode_attention, paged_decode_workspace,
                                        rope_kv_write, rope_kv_write_slots, write_kv_cache)
from .minimal_llama import LlamaConfig, LlamaWeights, llama_forward, precompute_rope


class PagedKVCache:
    """Per-layer K and V pools of shape [num_blocks, n_heads, block_size, head_dim]."""

    def __init__(self, config: LlamaConfig, num_blocks: int, block_size: int = 16, device="cuda"):
        shape = (num_blocks, config.n_heads, block_size, config.head_dim)
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.k = [torch.zeros(shape, dtype=config.dtype, device=device) for _ in range(config.n_layers)]
        self.v = [torch.zeros(shape, dtype=config.dtype, device=device) for _ in range(config.n_layers)]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


def slots_for_positions(table, positions, block_size: int):
    """Cache slots (block_id * block_size + offset) of token positions of one request."""
    t = torch.as_tensor(table, dtype=torch.int64)
    pos = torch.as_tensor(positions, dtype=torch.int64)
    return t[pos // block_size] * block_size + pos % block_size


@dataclass
class _Fused:
    """Per-layer projection weights held transposed ([out, in], in contiguous),
    the layout lsb_linear streams; ``.t()`` views serve the prefill GEMMs."""
    w_qkv_t: torch.Tensor
    w_gu_t: torch.Tensor
    w_o_t: torch.Tensor
    w_down_t: torch.Tensor


class PagedDecoder:
    """Runs prefill into the paged cache, then CUDA-graph greedy decode steps."""

    def __init__(self, weights: LlamaWeights, config: LlamaConfig, cache: PagedKVCache,
                 block_manager: BlockManager, max_batch: int, max_blocks_per_seq: int,
                 device="cuda", use_lsb_linear: bool = False):
        self.w, self.cfg, self.cache, self.bm = weights, config, cache, block_manager
        self.device = torch.device(device)
        self.S, self.MB = max_batch, max_blocks_per_seq
        self.fused = [_Fused(torch.cat([l.q_proj, l.k_proj, l.v_proj], dim=1).t().contiguous(),
                             torch.cat([l.gate_proj, l.up_proj], dim=1).t().contiguous(),
                             l.o_proj.t().contiguous(), l.down_proj.t().contiguous())
                      for l in weights.layers]
        self.lm_head_t = weights.lm_head.t().contiguous()
        # Decode projections on lsb_linear (weights packed once into its tile
        # layout) when asked for and it serves this model and batch; cuBLAS
        # otherwise. Off by default: at config 5's shapes cuBLAS is faster
        # (measured, see the design notes of lsb_linear).
        self.lsb_linear = (use_lsb_linear and config.dtype in (torch.bfloat16, torch.float16)
                           and max_batch <= LINEAR_MAX_ROWS)
        self._packed = {}
        if self.lsb_linear:
            for fz in self.fused:
                for w_t in (fz.w_qkv_t, fz.w_gu_t, fz.w_o_t, fz.w_down_t):
                    self._packed[id(w_t)] = pack_linear_weight(w_t)
            self._packed[id(self.lm_head_t)] = pack_linear_weight(self.lm_head_t)
        self.cos, self.sin = precompute_rope(config, self.device)
        S, Hd, H, D = max_batch, config.hidden_size, config.n_heads, config.head_dim
        dev = self.device
        self.tokens = torch.zeros(S, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(S, dtype=torch.int64, device=dev)
        self.context_lens = torch.zeros(S, dtype=torch.int32, device=dev)
        self.block_tables = torch.full((S, max_blocks_per_seq), -1, dtype=torch.int32, device=dev)
        self.zeros = torch.zeros(S, Hd, dtype=config.dtype, device=dev)
        self.attn_out = torch.empty(S, H, D, dtype=config.dtype, device=dev)
        self.q_rot = torch.empty(S, H, D, dtype=config.dtype, device=dev)
        self.act = torch.empty(S, config.intermediate_size, dtype=config.dtype, device=dev)
        self.ws = paged_decode_workspace((S, H, D), max_blocks_per_seq, cache.block_size, dev)
        self.graph = None
        self.requests: list = []

    # ------------------------------------------------------------ admission --
    def packed_prefill_supported(self) -> bool:
        return self.cfg.dtype in (torch.bfloat16, torch.float16) and self.cfg.head_dim in (64, 128)

    def admit(self, requests, max_new_tokens: int, packed: bool | None = None) -> torch.Tensor:
        """Allocates blocks, runs the prompts' prefill into the cache and returns
        the first greedy token of every request (int64 [len(requests)]).
        ``packed`` (default: when supported) prefills all prompts in one packed
        forward instead of one ``llama_forward`` per request."""
        assert len(requests) <= self.S
        bs = self.cache.block_size
        if packed is None:
            packed = self.packed_prefill_supported()
        first = []
        tables = []
        for r in requests:
            assert self.bm.can_allocate(r), f"not enough KV blocks for {r.request_id}"
            self.bm.allocate(r)
            # Reserve the decode blocks with the per-token append_slot sequence.
            n0 = len(r.output_token_ids)
            for _ in range(max_new_tokens + 1):
                r.output_token_ids.append(-1)
                self.bm.append_slot(r)
            del r.output_token_ids[n0:]
            table = self.bm.get_block_table(r)
            assert len(table) <= self.MB, "max_blocks_per_seq too small"
            tables.append(table)
            if not packed:
                first.append(self._prefill_one(r.prompt_token_ids, table))
        if packed:
            first = list(self.prefill_packed(requests, tables)) if requests else []
        self.requests = list(requests)
        nreq = len(requests)
        bt = self.bm.as_tensor(requests, self.MB)
        self.block_tables.fill_(-1)
        self.block_tables[:nreq].copy_(bt.to(self.device))
        first_t = torch.stack(first).to(torch.int64)
        self.tokens.zero_()
        self.tokens[:nreq].copy_(first_t)
        self.positions.zero_()
        self.positions[:nreq].copy_(torch.tensor([len(r.prompt_token_ids) for r in requests],
                                                 dtype=torch.int64, device=self.device))
        return first_t

    def _prefill_one(self, token_ids, table) -> torch.Tensor:
        """One sequence through ``llama_forward`` with its K/V sent to the cache
        slots of ``table``; returns its greedy next token (0-d int64)."""
        ids = torch.tensor([list(token_ids)], dtype=torch.int64, device=self.device)
        slots = slots_for_positions(table, range(ids.shape[1]), self.cache.block_size).to(self.device)

        def sink(li, k, v):
            write_kv_cache(k[0].transpose(0, 1), v[0].transpose(0, 1), self.cache.k[li],
                           self.cache.v[li], slots)

        logits = llama_forward(self.w, self.cfg, ids, causal=True, kv_sink=sink, last_only=True)
        return logits[0, -1].argmax(-1)

    def prefill(self, token_lists, tables) -> list:
        """Prefill of whole sequences (prompt plus any tokens generated before a
        preemption) into the cache slots of ``tables``; returns each one's greedy
        next token (host ints). Packed when supported, else one at a time."""
        if not token_lists:
            return []
        if self.packed_prefill_supported():
            return self.prefill_sequences(token_lists, tables).tolist()
        return [int(self._prefill_one(t, tb)) for t, tb in zip(token_lists, tables)]

    def prefill_packed(self, requests, tables) -> torch.Tensor:
        """``prefill_sequences`` over the prompts of ``requests``."""
        return self.prefill_sequences([r.prompt_token_ids for r in requests], tables)

    def prefill_sequences(self, token_lists, tables) -> torch.Tensor:
        """One forward over every token of ``token_lists`` (packed along the
        token axis), writing each token's K/V into its cache slot; returns the
        greedy next token of each sequence (int64 [len(token_lists)])."""
        assert self.packed_prefill_supported()
        cfg, bs, dev = self.cfg, self.cache.block_size, self.device
        H, D, Hd = cfg.n_heads, cfg.head_dim, cfg.hidden_size
        lens = [len(t) for t in token_lists]
        assert min(lens) > 0, "empty prompt"
        assert max(lens) <= cfg.max_seq_len, "sequence longer than the RoPE table"
        T = sum(lens)
        ids = torch.tensor([t for seq in token_lists for t in seq], dtype=torch.int64)
        positions = torch.cat([torch.arange(n, dtype=torch.int64) for n in lens])
        slots = torch.cat([slots_for_positions(tb, range(n), bs) for tb, n in zip(tables, lens)])
        cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
        ids, positions, slots, cu = (t.to(dev, non_blocking=True) for t in (ids, positions, slots, cu))
        residual = F.embedding(ids, self.w.embed_tokens)
        x = torch.zeros_like(residual)
        q_rot = torch.empty(T, H, D, dtype=cfg.dtype, device=dev)
        k_rot = torch.empty_like(q_rot)
        attn = torch.empty_like(q_rot)
        for li, layer in enumerate(self.w.layers):
            fz = self.fused[li]
            normed, residual = fused_add_rmsnorm(x, residual, layer.input_layernorm_weight, eps=cfg.rms_eps)
            qkv = (normed @ fz.w_qkv_t.t()).view(T, 3, H, D)
            rope_kv_write_slots(qkv, self.cos, self.sin, positions, slots, q_rot, k_rot,
                                self.cache.k[li], self.cache.v[li])
            flash_attention_varlen(q_rot, k_rot, qkv[:, 2], cu, max(lens), causal=True, out=attn)
            x = attn.view(T, Hd) @ layer.o_proj
            normed2, residual = fused_add_rmsnorm(x, residual, layer.post_attention_layernorm_weight,
                                                  eps=cfg.rms_eps)
            x = silu_and_mul(normed2 @ fz.w_gu_t.t()) @ layer.down_proj
        last = (cu[1:] - 1).long()
        final, _ = fused_add_rmsnorm(x[last].contiguous(), residual[last].contiguous(), self.w.norm_weight,
                                     eps=cfg.rms_eps)
        return (final @ self.w.lm_head).argmax(-1)

    # ------------------------------------------------------- slot decode --
    def decode_slots(self, slots, tokens, positions, tables, use_graph: bool = True) -> list:
        """One decode step for the sequences in batch rows ``slots``: row
        slots[i] processes tokens[i] at positions[i] with block table
        tables[i]; every other row is idle (no block table, so no cache write).
        Returns the greedy next token of each given slot (host ints). The
        CUDA graph is captured on first use, with every row idle.

        Host state lives in pinned buffers; a row's block table is rewritten
        only when another table takes the row, otherwise only its new
        entries are appended (block tables grow by appending)."""
        if use_graph and self.graph is None:
            self.block_tables.fill_(-1)
            self.capture()
        if not hasattr(self, "_h_bt"):
            self._h_tok = torch.zeros(self.S, dtype=torch.int64).pin_memory()
            self._h_pos = torch.zeros(self.S, dtype=torch.int64).pin_memory()
            self._h_bt = torch.full((self.S, self.MB), -1, dtype=torch.int32).pin_memory()
            self._row_src = [None] * self.S  # table list each row was written from
            self._row_len = [0] * self.S
        tok, pos, bt = self._h_tok.numpy(), self._h_pos.numpy(), self._h_bt.numpy()
        active = set(slots)
        for s_ in range(self.S):
            if s_ not in active and self._row_src[s_] is not None:
                bt[s_, :] = -1
                self._row_src[s_], self._row_len[s_] = None, 0
                tok[s_] = pos[s_] = 0
        for s_, t, p_, tb in zip(slots, tokens, positions, tables):
            assert len(tb) <= self.MB, "block table longer than max_blocks_per_seq"
            assert p_ < self.cfg.max_seq_len, "position beyond the RoPE table"
            tok[s_], pos[s_] = t, p_
            n0 = self._row_len[s_]
            if self._row_src[s_] is not tb or len(tb) < n0:
                bt[s_, :] = -1
                n0 = 0
            if len(tb) > n0:
                bt[s_, n0:len(tb)] = tb[n0:]
            self._row_src[s_], self._row_len[s_] = tb, len(tb)
        self.tokens.copy_(self._h_tok, non_blocking=True)
        self.positions.copy_(self._h_pos, non_blocking=True)
        self.block_tables.copy_(self._h_bt, non_blocking=True)
        if use_graph:
            self.graph.replay()
        else:
            self.step()
        nxt = self.tokens.cpu()  # also orders the next step's host writes after these copies
        return [int(nxt[s_]) for s_ in slots]

    # ----------------------------------------------------------------- step --
    def _proj(self, x: torch.Tensor, w_t: torch.Tensor) -> torch.Tensor:
        """x @ w for a decode batch, with w held transposed."""
        if self.lsb_linear:
            return linear(x, self._packed[id(w_t)])
        return x @ w_t.t()

    def step(self) -> torch.Tensor:
        """One greedy decode step over the static buffers; returns next tokens [S]."""
        cfg, S, bs = self.cfg, self.S, self.cache.block_size
        H, D, Hd, I = cfg.n_heads, cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
        pos = self.positions
        residual = F.embedding(self.tokens, self.w.embed_tokens)
        x = self.zeros
        mm = self._proj
        for li, layer in enumerate(self.w.layers):
            fz = self.fused[li]
            normed, residual = fused_add_rmsnorm(x, residual, layer.input_layernorm_weight, eps=cfg.rms_eps)
            qkv = mm(normed, fz.w_qkv_t).view(S, 3, H, D)
            # RoPE at each sequence's position + K/V into its cache slot, fused
            # (also sets context_lens = positions + 1).
            q = rope_kv_write(qkv, self.cos, self.sin, pos, self.block_tables, self.q_rot,
                              self.cache.k[li], self.cache.v[li], self.context_lens)
            attn = paged_decode_attention(q, self.cache.k[li], self.cache.v[li], self.block_tables,
                                          self.context_lens, out=self.attn_out, workspace=self.ws)
            x = mm(attn.view(S, Hd), fz.w_o_t)
            normed2, residual = fused_add_rmsnorm(x, residual, layer.post_attention_layernorm_weight,
                                                  eps=cfg.rms_eps)
            gu = mm(normed2, fz.w_gu_t)
            x = mm(silu_and_mul(gu, out=self.act), fz.w_down_t)
        final, _ = fused_add_rmsnorm(x, residual, self.w.norm_weight, eps=cfg.rms_eps)
        logits = mm(final, self.lm_head_t)
        # Next token of every row (argmax) into self.tokens, positions + 1.
        greedy_next(logits, self.tokens, self.positions)
        return self.tokens

    def capture(self, warmup: int = 3):
        """Side-stream warm-up, then capture one step into a CUDA graph.

        Warm-up steps advance the positions and overwrite cache slots beyond
        the prompt, so the state is saved and restored around them."""
        saved = (self.tokens.clone(), self.positions.clone())
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.step()
                self.tokens.copy_(saved[0]); self.positions.copy_(saved[1])
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.tokens.copy_(saved[0]); self.positions.copy_(saved[1])
        self.graph = g
        return g

    def decode(self, num_steps: int, use_graph: bool = True) -> torch.Tensor:
        """Runs num_steps steps; returns int64 [S, num_steps] generated tokens (on device)."""
        hist = torch.empty(self.S, num_steps, dtype=torch.int64, device=self.device)
        if use_graph and self.graph is None:
            self.capture()
        for i in range(num_steps):
            if use_graph:
                self.graph.replay()
            else:
                self.step()
            hist[:, i].copy_(self.tokens)
        return hist

    def generate(self, requests, max_new_tokens: int, use_graph: bool = True):
        """First token from prefill plus max_new_tokens - 1 decode steps, written back
        to each request's output_token_ids; returns the token lists."""
        first = self.admit(requests, max_new_tokens)
        hist = self.decode(max_new_tokens - 1, use_graph=use_graph) if max_new_tokens > 1 else None
        out = []
        first = first.tolist()
        h = hist.cpu().tolist() if hist is not None else None
        for i, r in enumerate(requests):
            toks = [first[i]] + (h[i] if h is not None else [])
            r.output_token_ids.extend(toks)
            out.append(toks)
        return out
