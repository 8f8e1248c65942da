"""In-house rollout engine (replaces vLLM / MCore inference in the reference).

Reference behaviour: ``VllmGenerationWorkerImpl.generate``
(``nemo_rl/models/generation/vllm/vllm_worker.py:1120``), the MCore dynamic engine
(``nemo_rl/models/generation/megatron/megatron_worker.py:1396``, paged KV with
``block_size_tokens: 256``), sleep / wake of KV memory for colocation
(``vllm_worker.py:1635,1663``) and CUDA-graph decode (``enforce_eager: False``).

Design (B200-first)
-------------------
* Weights are the trainer's own bf16 parameters (colocated by construction),
  so a refit after an optimizer step costs nothing here; an fp8 rollout copy
  is re-quantised by the refit kernel when requested.
* Paged KV cache in one allocation ``[L, 2, blocks, block, nkv, hd]``; blocks
  are handed out per sequence up front for ``prompt + max_new_tokens``.
* Prefill runs all prompts packed (THD) through the varlen attention kernel
  and writes K/V to the cache.
* Decode runs ENTIRELY on the device: one CUDA graph per batch bucket does
  slot computation, the model step, LM head, sampling, the output write and
  stop-token / length bookkeeping.  The host only replays the graph and reads
  a single "all done" flag every ``sync_every`` steps.  Finished rows are
  compacted into a smaller bucket when the active set halves.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.models.transformer import KVCache, TransformerLM
from rl_b200.ops._ext import add_launches, launch_count
from rl_b200.ops.sampling import sample_tokens

__all__ = ["RolloutEngine"]


def _buckets(max_bs: int) -> list[int]:
    out, b = [], 1
    while b < max_bs:
        out.append(b)
        b *= 2
    out.append(max_bs)
    return sorted(set(out))


class _DecodeState:
    """Static device buffers for one batch bucket (graph inputs / outputs)."""

    def __init__(self, B: int, max_blocks: int, max_new: int, device):
        i32, i64 = torch.int32, torch.int64
        self.B = B
        self.tokens = torch.zeros(B, dtype=i64, device=device)
        self.positions = torch.zeros(B, dtype=i32, device=device)
        self.seq_lens = torch.zeros(B, dtype=i32, device=device)
        self.slot = torch.zeros(B, dtype=i64, device=device)
        self.block_tables = torch.zeros(B, max_blocks, dtype=i32, device=device)
        self.done = torch.ones(B, dtype=torch.bool, device=device)
        self.gen_len = torch.zeros(B, dtype=i32, device=device)
        self.max_new = torch.zeros(B, dtype=i32, device=device)
        self.step = torch.zeros(1, dtype=i64, device=device)
        self.rng_offset = torch.zeros(1, dtype=i64, device=device)
        self.out_tokens = torch.zeros(B, max_new + 1, dtype=i64, device=device)
        self.out_logprobs = torch.zeros(B, max_new + 1, dtype=torch.float32, device=device)
        self.next_tokens = torch.zeros(B, dtype=i64, device=device)
        self.next_logprobs = torch.zeros(B, dtype=torch.float32, device=device)
        self.stop = torch.full((8,), -1, dtype=i64, device=device)  # stop-token ids (graph input)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.native_launches = 0


class RolloutEngine:
    def __init__(self, model: TransformerLM, gen_cfg: dict, max_num_seqs: int = 256, max_model_len: int = 2048,
                 block_size: int = 256, kv_dtype: Optional[torch.dtype] = None, use_cuda_graphs: bool = True,
                 seed: int = 0, sync_every: int = 32):
        self.model = model
        self.cfg = dict(gen_cfg)
        self.device = model.device
        self.max_num_seqs = max_num_seqs
        self.max_model_len = max_model_len
        self.block_size = block_size
        self.kv_dtype = kv_dtype or model.dtype
        # expert-parallel MoE decode sizes its token exchange on the host every step
        # (row totals per expert owner), which a captured graph cannot replay
        self.use_cuda_graphs = use_cuda_graphs and self.device.type == "cuda" and model.ps.ep_size == 1
        self.seed = seed
        self.sync_every = sync_every
        self.kv: Optional[KVCache] = None
        # speculative decoding: a small draft LM proposes `num_spec` tokens per
        # round, the target verifies them in one batched forward
        self.draft: Optional[TransformerLM] = None
        self.draft_kv: Optional[KVCache] = None
        self.num_spec = int((self.cfg.get("speculative") or {}).get("num_speculative_tokens", 0) or 0)
        self.spec_stats = {"rounds": 0, "emitted": 0, "proposed": 0}
        self.max_blocks_per_seq = math.ceil((max_model_len + self.num_spec + 1) / block_size)
        self._states: dict[int, _DecodeState] = {}
        self._graph_pool = None
        self.calls = 0
        self.stats: dict = {}
        # optional callable returning a device buffer whose bytes the KV cache may
        # occupy while generating (colocated trainer: its idle gradient arena)
        self.kv_arena = None
        # True once the KV cache has written into the arena (the owner must reset it)
        self.arena_dirty = False
        # "thread_local" when another thread keeps launching work while decode
        # graphs are captured (async GRPO's rollout thread)
        self.capture_error_mode = "global"
        # router replay (R3): record the experts every MoE layer picks for every
        # processed token and return them as "routed_experts" [B, S, layers, k]
        # (-1 where no route exists: padding and the last sampled token)
        self.record_routes = False
        self._route_steps: Optional[list] = None
        # fp8 KV cache: per-layer (k, v) scales from calibrate_qkv_fp8_scales
        self.kv_scales: Optional[tuple] = None
        # score centering: record the sampler's top-k (ids, log-probs) of every
        # generated token's distribution ("sampler_topk_token_ids / _logprobs")
        self.record_sampler_topk = 0
        self._topk_steps: Optional[list] = None

    # ------------------------------------------------------------ lifecycle
    def prepare_for_generation(self, num_seqs: Optional[int] = None) -> bool:
        """Allocate (wake) the KV cache."""
        if self.kv is None:
            n = num_seqs or self.max_num_seqs
            blocks = n * self.max_blocks_per_seq + 1
            arena = self.kv_arena() if self.kv_arena is not None else None
            self.kv = KVCache(self.model.cfg.num_layers, blocks, self.block_size, self.model.nkv, self.model.hd,
                              self.kv_dtype, self.device, arena=arena)
            if self.kv_scales is not None:
                self.kv.k_scales, self.kv.v_scales = list(self.kv_scales[0]), list(self.kv_scales[1])
            self.arena_dirty = self.arena_dirty or (arena is not None)
            self._kv_capacity_seqs = n
            if self.draft is not None:
                d = self.draft
                self.draft_kv = KVCache(d.cfg.num_layers, blocks, self.block_size, d.nkv, d.hd, self.kv_dtype,
                                        self.device)
            sig = (self.kv.storage.data_ptr(), tuple(self.kv.storage.shape))
            if sig != getattr(self, "_kv_sig", None):
                self._drop_graphs()  # captured graphs point at the old cache
            self._kv_sig = sig
        return True

    def set_kv_scales(self, k_scales: list, v_scales: list) -> None:
        """Per-layer fp8 KV-cache scales (cache value = k / k_scale); captured
        decode graphs bake the scales in, so they are dropped."""
        self.kv_scales = (list(k_scales), list(v_scales))
        if self.kv is not None:
            self.kv.k_scales, self.kv.v_scales = list(k_scales), list(v_scales)
        self._drop_graphs()

    def _drop_graphs(self) -> None:
        for st in self._states.values():
            st.graph = None
        self._states.clear()
        self._graph_pool = None

    def set_draft(self, draft, num_speculative_tokens: int) -> None:
        """Enable speculative decoding with ``draft`` proposing ``num_speculative_tokens``
        tokens per round (the KV caches are re-created at the next prepare): a
        small LM (its own embedding) or an Eagle3 head (``rl_b200.models.eagle3``,
        fed the target's hidden features) or a block drafter (``DFlashDraft``)."""
        self.draft = draft
        # "dflash": a block drafter (one forward proposes the whole block);
        # "eagle3": a feature-fed head drafting token by token; "lm": a small LM
        self.draft_kind = "dflash" if hasattr(draft, "propose") else ("eagle3" if hasattr(draft, "fuse") else "lm")
        self.num_spec = int(num_speculative_tokens)
        self.max_blocks_per_seq = math.ceil((self.max_model_len + self.num_spec + 1) / self.block_size)
        self.finish_generation()
        self._drop_graphs()
        self._kv_sig = None

    def finish_generation(self) -> bool:
        """Release (sleep) the KV cache so training gets the memory back.

        When the cache lives in a persistent arena its address is stable across
        steps, so the captured decode graphs are kept and replayed next time;
        otherwise they are dropped with the cache."""
        self.kv = None
        self.draft_kv = None
        if self.kv_arena is None:
            self._drop_graphs()
            self._kv_sig = None
        # No empty_cache(): the freed KV blocks stay mapped in the caching allocator and
        # are reused by the trainer's gradient buffer (and vice versa) every step,
        # instead of being unmapped and re-mapped (seconds per step for ~45 GB).
        return True

    def invalidate_kv_cache(self) -> bool:
        return True  # no prefix caching across refits: nothing to invalidate

    def update_weights_from_training(self) -> None:
        """Colocated refit: the engine reads the trainer's parameters directly."""
        return None

    # ------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, data: BatchedDataDict, greedy: bool = False, max_new_tokens: Optional[int] = None
                 ) -> BatchedDataDict:
        input_ids: torch.Tensor = data["input_ids"]
        lengths: torch.Tensor = data["input_lengths"].to(torch.int64)
        B, S = input_ids.shape
        cfg = self.cfg
        max_new = int(max_new_tokens if max_new_tokens is not None else cfg.get("max_new_tokens", 16))
        max_new = max(0, min(max_new, self.max_model_len - int(lengths.max())))
        pad_id = int(cfg.get("pad_token_id", 0))
        temperature = 0.0 if greedy else float(cfg.get("temperature", 1.0))
        top_k = cfg.get("top_k")
        top_p = float(cfg.get("top_p", 1.0) or 1.0)
        stop_ids = list(cfg.get("stop_token_ids") or [])
        out_ids = torch.full((B, S + max_new), pad_id, dtype=torch.int64)
        out_lp = torch.zeros((B, S + max_new), dtype=torch.float32)
        out_ids[:, :S] = input_ids.cpu()
        gen_lens = torch.zeros(B, dtype=torch.int64)
        self.calls += 1
        if max_new == 0 or B == 0:
            return self._pack_outputs(out_ids, out_lp, lengths, gen_lens, pad_id, max_new)

        self.prepare_for_generation(max(B, getattr(self, "_kv_capacity_seqs", 0)))
        if B > self._kv_capacity_seqs:
            self.finish_generation()
            self.prepare_for_generation(B)
        dev = self.device
        bs = self.block_size
        nblk = self.max_blocks_per_seq
        block_tables = (torch.arange(B * nblk, dtype=torch.int32).view(B, nblk) + 1).to(dev)  # block 0 = scratch

        # ---- prefill (packed prompts) ----
        lens_l = lengths.tolist()
        recording = self.record_routes and self.model.cfg.is_moe
        topk_rec = int(self.record_sampler_topk or 0)
        spec = self._spec_enabled(top_k, top_p) and not recording and not topk_rec
        mg = cfg.get("mcore_generation_config") or {}
        # identical prompts (a GRPO group's samples) are prefilled once; their KV
        # blocks are copied to the other rows of the group
        dedup = bool(mg.get("enable_prefix_caching", True)) and not recording
        # prefill in passes of at most max_tokens tokens (whole sequences), which
        # bounds the prefill activations; not under expert parallelism, whose
        # collectives need the same pass count on every rank
        ep = getattr(getattr(self.model, "ps", None), "ep_size", 1)
        chunk_tokens = int(mg.get("max_tokens", 16384)) if (mg.get("enable_chunked_prefill", True)
                                                             and not recording and ep <= 1) else 0
        rep, inv = self._unique_prompts(input_ids, lens_l) if dedup else (list(range(B)), list(range(B)))
        if recording:
            self.model.router_record = {}
        h_parts = []
        self._eagle_fprev_rows = {}
        for rows in self._prefill_passes(rep, lens_l, chunk_tokens):
            h_parts.append(self._prefill_rows(input_ids, rows, lens_l, block_tables, spec))
        h = torch.cat(h_parts) if len(h_parts) > 1 else h_parts[0]
        if len(rep) < B:
            self._copy_prompt_blocks(rep, inv, lens_l, block_tables, spec)
            h = h[torch.tensor(inv, device=h.device)]
        if self._eagle_fprev_rows:
            self._eagle_fprev = torch.stack([self._eagle_fprev_rows[rep[u]] for u in inv])
        self.stats_last_prefill = {"prompts": B, "prefilled": len(rep), "passes": len(h_parts),
                                   "tokens": int(sum(lens_l[r] for r in rep))}
        prefill_routes = self._take_routes() if recording else None
        self._route_steps = [] if recording else None
        logits = self.model.logits_infer(h)
        self._topk_steps = [self._sampler_topk(logits, temperature, topk_rec)] if topk_rec else None
        gen = None
        if dev.type == "cpu":
            gen = torch.Generator().manual_seed(self.seed * 7919 + self.calls)
        tok0, lp0 = sample_tokens(logits, temperature if temperature > 0 else 1.0,
                                  1 if temperature == 0 else top_k, top_p, seed=self.seed,
                                  offset=self.calls * (1 << 24), generator=gen)
        if temperature == 0:
            lp0 = torch.zeros_like(lp0)

        # ---- decode ----
        if recording or topk_rec:
            # routes are read back after every step: eager decode (no graphs, no speculation)
            try:
                tokens_all, lps_all, glen = self._decode_loop(tok0, lp0, lengths.to(dev), block_tables, max_new,
                                                              temperature, top_k, top_p, stop_ids, gen, eager=True)
            finally:
                self.model.router_record = None
        elif spec:
            tokens_all, lps_all, glen = self._spec_decode_loop(tok0, lp0, lengths.to(dev), block_tables, max_new,
                                                               temperature, stop_ids)
        else:
            tokens_all, lps_all, glen = self._decode_loop(tok0, lp0, lengths.to(dev), block_tables, max_new,
                                                          temperature, top_k, top_p, stop_ids, gen)
        glen_c = glen.cpu().to(torch.int64)
        toks_c = tokens_all.cpu()
        lps_c = lps_all.cpu()
        for b in range(B):
            n = int(glen_c[b])
            L = lens_l[b]
            out_ids[b, L: L + n] = toks_c[b, :n]
            out_lp[b, L: L + n] = lps_c[b, :n]
        out = self._pack_outputs(out_ids, out_lp, lengths, glen_c, pad_id, max_new)
        if recording:
            out["routed_experts"] = self._assemble_routes(prefill_routes, lens_l, glen_c, out["output_ids"].shape[1])
            self._route_steps = None
        if topk_rec:
            W = out["output_ids"].shape[1]
            ids = torch.zeros(B, W, topk_rec, dtype=torch.int64)
            lps = torch.zeros(B, W, topk_rec, dtype=torch.float32)
            steps = [(a.cpu(), b.cpu()) for a, b in self._topk_steps]
            for b in range(B):
                L, n = lens_l[b], int(glen_c[b])
                for s_ in range(min(n, len(steps))):  # generated token s_ came from distribution s_
                    ids[b, L + s_], lps[b, L + s_] = steps[s_][0][b], steps[s_][1][b]
            out["sampler_topk_token_ids"], out["sampler_topk_logprobs"] = ids, lps
            self._topk_steps = None
        return out

    @staticmethod
    def _unique_prompts(input_ids: torch.Tensor, lens: list) -> tuple[list[int], list[int]]:
        """(first row of each distinct prompt, for every row the index of its
        prompt in that list)."""
        seen: dict = {}
        rep, inv = [], []
        ids = input_ids.cpu()
        for b, L in enumerate(lens):
            key = (L, ids[b, :L].numpy().tobytes())
            if key not in seen:
                seen[key] = len(rep)
                rep.append(b)
            inv.append(seen[key])
        return rep, inv

    @staticmethod
    def _prefill_passes(rows: list[int], lens: list, max_tokens: int) -> list[list[int]]:
        """Consecutive runs of ``rows`` of at most ``max_tokens`` prompt tokens (a
        longer prompt runs alone); one pass when ``max_tokens`` is 0."""
        if max_tokens <= 0:
            return [rows]
        out, cur, n = [], [], 0
        for r in rows:
            if cur and n + lens[r] > max_tokens:
                out.append(cur)
                cur, n = [], 0
            cur.append(r)
            n += lens[r]
        if cur:
            out.append(cur)
        return out

    def _prefill_rows(self, input_ids: torch.Tensor, rows: list[int], lens: list, block_tables: torch.Tensor,
                      spec: bool) -> torch.Tensor:
        """Prefill the prompts of ``rows`` into their KV blocks; returns the last
        position's hidden state of each, ``[len(rows), H]``."""
        dev = self.device
        bs = self.block_size
        rl = [lens[r] for r in rows]
        flat = torch.cat([input_ids[r, :L].cpu() for r, L in zip(rows, rl)])
        if dev.type == "cuda":
            flat = flat.pin_memory()  # the step's inputs cross PCIe once, from pinned memory
        flat = flat.to(dev, non_blocking=True)
        positions = torch.cat([torch.arange(L, dtype=torch.int32) for L in rl]).to(dev)
        cu = torch.zeros(len(rows) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(rl), 0)
        cu_d = cu.to(dev)
        seq_row = torch.repeat_interleave(torch.tensor(rows), torch.tensor(rl)).to(dev)
        slot = (block_tables[seq_row, (positions // bs).long()].long() * bs + (positions % bs).long())
        last_idx = (cu[1:] - 1).to(dev).long()
        eagle = spec and getattr(self, "draft_kind", "lm") in ("eagle3", "dflash")
        if eagle:  # feature-fed drafts read the target's hidden features of every prompt position
            self.model.capture_layers, self.model.captured = self.draft.aux_layers, None
        try:
            h = self.model.forward_prefill(flat, positions, cu_d, max(rl), self.kv, slot, last_idx)
            feats = (torch.cat([self.model.captured[i] for i in self.draft.aux_layers], -1) if eagle else None)
        finally:
            if eagle:
                self.model.capture_layers, self.model.captured = None, None
        if eagle:
            from rl_b200.models.eagle3 import shift_features

            with torch.no_grad():
                if self.draft_kind == "eagle3":  # the block drafter keeps no draft cache
                    self.draft.prefill(self.model.embed_full(flat), shift_features(feats, cu_d), positions, cu_d,
                                       max(rl), self.draft_kv, slot, last_idx)
                for r, f in zip(rows, self.draft.fuse(feats[last_idx])):
                    self._eagle_fprev_rows[r] = f  # feature of each prompt's last position
        elif spec:
            self.draft.forward_prefill(flat, positions, cu_d, max(rl), self.draft_kv, slot, last_idx)
        return h

    def _copy_prompt_blocks(self, rep: list[int], inv: list[int], lens: list, block_tables: torch.Tensor,
                            spec: bool) -> None:
        """Give every duplicate row the KV blocks of its prompt's prefilled row."""
        bs = self.block_size
        src, dst = [], []
        for b, u in enumerate(inv):
            r = rep[u]
            if r == b:
                continue
            nb = -(-lens[b] // bs)
            src.append(block_tables[r, :nb])
            dst.append(block_tables[b, :nb])
        if not src:
            return
        src_t, dst_t = torch.cat(src).long(), torch.cat(dst).long()
        for cache in ([self.kv, self.draft_kv] if spec else [self.kv]):
            st = cache.storage
            if st.element_size() == 1:
                st = st.view(torch.uint8)  # fp8 caches: copy the bytes
            for layer in range(st.shape[0]):  # per layer: the gathered blocks stay small
                for kv in range(2):
                    t = st[layer, kv]
                    t.index_copy_(0, dst_t, t.index_select(0, src_t))

    @staticmethod
    def _sampler_topk(logits: torch.Tensor, temperature: float, k: int):
        """Top-k (ids, log-probs) of the sampling distribution (temperature-scaled)."""
        lp = torch.log_softmax(logits.float() / (temperature if temperature > 0 else 1.0), -1)
        v, i = lp.topk(k, -1)
        return i, v

    def _take_routes(self) -> torch.Tensor:
        """The routes recorded by the last forward, ``[T, layers, k]``; resets the record."""
        rec = self.model.router_record
        out = torch.stack([rec[i] for i in sorted(rec)], 1)
        self.model.router_record = {}
        return out

    def _assemble_routes(self, prefill: torch.Tensor, lens: list, glen: torch.Tensor, width: int) -> torch.Tensor:
        """Per-sequence routes ``[B, width, layers, k]``: prompt positions from the
        prefill, position ``L + s - 1`` from decode step ``s`` (the token fed at
        that step); the last sampled token was never fed and stays -1."""
        B = len(lens)
        nl, k = prefill.shape[1], prefill.shape[2]
        out = torch.full((B, width, nl, k), -1, dtype=prefill.dtype)
        pre = prefill.cpu()
        steps = [t.cpu() for t in self._route_steps]
        off = 0
        for b in range(B):
            L, n = lens[b], int(glen[b])
            out[b, :L] = pre[off:off + L]
            off += L
            for s in range(1, n):
                out[b, L + s - 1] = steps[s - 1][b]
        return out

    def _spec_enabled(self, top_k, top_p) -> bool:
        # rejection sampling verifies against the full distributions: no top-k / top-p filtering
        return (self.draft is not None and self.num_spec > 0 and self.draft_kv is not None
                and not top_k and (top_p is None or top_p >= 1.0))

    def _spec_decode_loop(self, tok0, lp0, lengths, block_tables, max_new, temperature, stop_ids):
        """Speculative decoding (eager): per round the draft proposes k tokens, the
        target scores [last, d_1..d_k] at positions L..L+k in ONE batched decode
        forward (row (b, j) sees keys up to L+j), and ``spec_verify`` accepts a
        prefix and adds a correction.  At most k tokens are emitted per round (a
        full acceptance's bonus token is left for the next round, which keeps
        the draft's cache gap-free); the output distribution is the target's."""
        from rl_b200.ops.sampling import sample_tokens
        from rl_b200.ops.spec_decode import spec_verify

        dev = self.device
        B = tok0.shape[0]
        k = self.num_spec
        bs = self.block_size
        cap = max_new + k + 1
        toks = torch.zeros(B, cap, dtype=torch.int64, device=dev)
        lps = torch.zeros(B, cap, dtype=torch.float32, device=dev)
        toks[:, 0], lps[:, 0] = tok0, lp0
        stop = torch.tensor(stop_ids if stop_ids else [-1], dtype=torch.int64, device=dev)
        glen = torch.ones(B, dtype=torch.int64, device=dev)
        done = torch.isin(tok0, stop) | (glen >= max_new)
        last = tok0.clone()
        pos0 = lengths.to(torch.int64).clone()       # position of `last`
        ar = torch.arange(k + 1, device=dev)
        bt_rows = block_tables.repeat_interleave(k + 1, 0)
        temp = temperature if temperature > 0 else 0.0
        rnd = 0
        kind = getattr(self, "draft_kind", "lm")
        eagle = kind in ("eagle3", "dflash")
        fprev = self._eagle_fprev if eagle else None  # target feature of the position before `last`
        maxlen = self.max_model_len + k + 1
        while not bool(done.all()):
            # 1. draft proposals (rows of finished sequences run too; results are ignored)
            x = last
            drafts, dlogits = [], []
            f = fprev
            block = self.draft.propose(self.model.embed_full(x), f, k).view(B, k, -1) if kind == "dflash" else None
            for j in range(k):
                if block is not None:  # the block's rows were proposed together: sample each
                    lg = block[:, j]
                    x, _ = sample_tokens(lg, temp if temp > 0 else 1.0, 1 if temp == 0 else None, 1.0,
                                         seed=self.seed + 17, offset=(self.calls << 24) + rnd * (k + 1) + j)
                    drafts.append(x)
                    dlogits.append(lg)
                    continue
                p = (pos0 + j).to(torch.int32)
                slot = block_tables.gather(1, (p // bs).long().unsqueeze(1)).squeeze(1).long() * bs + (p % bs).long()
                if eagle:  # later proposals feed back the draft's own hidden as the feature
                    f = self.draft.step(self.model.embed_full(x), f, p, self.draft_kv, block_tables, p + 1, slot,
                                        maxlen)
                    h = f
                else:
                    h = self.draft.forward_decode(x, p, self.draft_kv, block_tables, p + 1, slot, maxlen)
                lg = self.draft.logits_infer(h)
                x, _ = sample_tokens(lg, temp if temp > 0 else 1.0, 1 if temp == 0 else None, 1.0, seed=self.seed + 17,
                                     offset=(self.calls << 24) + rnd * (k + 1) + j)
                drafts.append(x)
                dlogits.append(lg)
            dr = torch.stack(drafts, 1)
            # 2. target verify of [last, d_1..d_k] at positions pos0 .. pos0+k
            rows_tok = torch.cat([last.unsqueeze(1), dr], 1).reshape(-1)
            rows_pos = (pos0.unsqueeze(1) + ar).reshape(-1).to(torch.int32)
            slot = bt_rows.gather(1, (rows_pos // bs).long().unsqueeze(1)).squeeze(1).long() * bs + (rows_pos % bs).long()
            if eagle:
                self.model.capture_layers, self.model.captured = self.draft.aux_layers, None
            try:
                h = self.model.forward_decode(rows_tok, rows_pos, self.kv, bt_rows, rows_pos + 1, slot, maxlen)
                vfeats = (torch.cat([self.model.captured[i] for i in self.draft.aux_layers], -1).view(B, k + 1, -1)
                          if eagle else None)
            finally:
                if eagle:
                    self.model.capture_layers, self.model.captured = None, None
            tl = self.model.logits_infer(h).view(B, k + 1, -1)
            out, n, olp = spec_verify(tl, torch.stack(dlogits, 1), dr, temp, seed=self.seed,
                                      offset=(self.calls << 20) + rnd)
            n = torch.clamp(n.to(torch.int64), max=k)
            # 3. append the emitted tokens (cut at a stop token / the length budget)
            valid = ar[:k].unsqueeze(0) < n.unsqueeze(1)
            is_stop = torch.isin(out[:, :k], stop) & valid
            first_stop = torch.where(is_stop.any(1), is_stop.float().argmax(1) + 1, n)
            room = (max_new - glen).clamp_min(0)
            take = torch.minimum(torch.minimum(n, first_stop), room)
            take = torch.where(done, torch.zeros_like(take), take)
            col = glen.unsqueeze(1) + ar[:k].unsqueeze(0)
            keep = ar[:k].unsqueeze(0) < take.unsqueeze(1)
            # columns glen..glen+k-1 < cap are distinct per row: rewrite kept slots only
            toks.scatter_(1, col, torch.where(keep, out[:, :k], toks.gather(1, col)))
            lps.scatter_(1, col, torch.where(keep, olp[:, :k], lps.gather(1, col)))
            glen = glen + take
            newly = (take > 0) & (first_stop <= take) & is_stop.any(1)
            done = done | newly | (glen >= max_new)
            last = torch.where(take > 0, out.gather(1, (take - 1).clamp_min(0).unsqueeze(1)).squeeze(1), last)
            if eagle:
                # the next round starts from the verified feature of the position before the
                # new `last`, and the draft cache entries of the accepted positions are
                # rewritten from verified features (proposals used the draft's own)
                rows_b = torch.arange(B, device=dev)
                f_new = self.draft.fuse(vfeats[rows_b, (take - 1).clamp_min(0)])
                fprev = torch.where((take > 0).unsqueeze(1), f_new, fprev)
                if k > 1 and kind == "eagle3":
                    fx_tok = out[:, : k - 1].reshape(-1)
                    fx_pos = (pos0.unsqueeze(1) + ar[1:k]).reshape(-1).to(torch.int32)
                    bt_fx = block_tables.repeat_interleave(k - 1, 0)
                    fx_slot = bt_fx.gather(1, (fx_pos // bs).long().unsqueeze(1)).squeeze(1).long() * bs + \
                        (fx_pos % bs).long()
                    self.draft.step(self.model.embed_full(fx_tok), self.draft.fuse(vfeats[:, : k - 1].reshape(B * (k - 1), -1)),
                                    fx_pos, self.draft_kv, bt_fx, fx_pos + 1, fx_slot, maxlen)
            pos0 = pos0 + take
            self.spec_stats["rounds"] += 1
            self.spec_stats["proposed"] += int(k * B)
            rnd += 1
        self.spec_stats["emitted"] += int(glen.sum())
        return toks[:, :max_new], lps[:, :max_new], glen.to(torch.int32)

    def _pack_outputs(self, out_ids, out_lp, lengths, gen_lens, pad_id, max_new) -> BatchedDataDict:
        unpadded = lengths.cpu() + gen_lens
        width = int(unpadded.max()) if len(unpadded) else out_ids.shape[1]
        width = max(width, 1)
        return BatchedDataDict({
            "output_ids": out_ids[:, :width].contiguous(),
            "logprobs": out_lp[:, :width].contiguous(),
            "generation_lengths": gen_lens.clone(),
            "unpadded_sequence_lengths": unpadded,
            "truncated": gen_lens >= max_new,
        })

    def _decode_loop(self, tok0, lp0, lengths, block_tables, max_new, temperature, top_k, top_p, stop_ids, gen,
                     eager: bool = False):
        dev = self.device
        B = tok0.shape[0]
        stop = torch.tensor(stop_ids if stop_ids else [-1], dtype=torch.int64, device=dev)
        # Global outputs (original row order)
        tokens_all = torch.zeros(B, max_new, dtype=torch.int64, device=dev)
        lps_all = torch.zeros(B, max_new, dtype=torch.float32, device=dev)
        tokens_all[:, 0] = tok0
        lps_all[:, 0] = lp0
        glen = torch.ones(B, dtype=torch.int32, device=dev)
        done0 = torch.isin(tok0, stop) | (glen >= max_new)
        active_rows = torch.nonzero(~done0).flatten()
        if active_rows.numel() == 0:
            return tokens_all, lps_all, glen
        if self.device.type != "cuda" or not self.use_cuda_graphs or eager:
            return self._decode_eager(tokens_all, lps_all, glen, tok0, lengths, block_tables, max_new, temperature,
                                      top_k, top_p, stop, gen, done0)
        rows = active_rows
        step_done = 1
        while rows.numel() > 0 and step_done < max_new:
            nb = next(b for b in _buckets(self.max_num_seqs) if b >= rows.numel()) \
                if rows.numel() <= self.max_num_seqs else rows.numel()
            st = self._state(nb, max_new, (temperature, top_k, top_p))
            n = rows.numel()
            st.stop.fill_(-1)
            st.stop[: min(len(stop_ids), st.stop.numel())] = stop[: st.stop.numel()] if stop_ids else -1
            st.done.fill_(True)
            st.done[:n] = False
            st.tokens.zero_()
            st.tokens[:n] = tokens_all[rows, step_done - 1]
            st.positions.zero_()
            st.positions[:n] = (lengths[rows] + step_done - 1).to(torch.int32)
            st.block_tables.zero_()
            st.block_tables[:n] = block_tables[rows]
            st.gen_len.zero_()
            st.gen_len[:n] = glen[rows]
            st.max_new.fill_(max_new)
            st.step.fill_(0)
            # the random stream depends on (call, step) through this device offset, so a
            # replayed graph draws fresh noise on every generate() call and step
            st.rng_offset.fill_(self.calls * (1 << 24) + step_done + 1)
            st.out_tokens.zero_()
            st.out_logprobs.zero_()
            if st.graph is None:
                self._capture(st, temperature, top_k, top_p, st.stop)
            k = 0
            while True:
                st.graph.replay()
                add_launches(st.native_launches)
                k += 1
                step_done_k = step_done + k
                if step_done_k >= max_new:
                    break
                if k % self.sync_every == 0:
                    remaining = int((~st.done[:n]).sum().item())
                    if remaining == 0:
                        break
                    if remaining <= n // 2 and nb > 1:
                        break  # compact into a smaller bucket
            # copy back this segment
            seg_tok = st.out_tokens[:n, :k]
            seg_lp = st.out_logprobs[:n, :k]
            cols = torch.arange(step_done, step_done + k, device=dev).clamp_max(max_new - 1)
            tokens_all[rows.unsqueeze(1), cols.unsqueeze(0)] = seg_tok
            lps_all[rows.unsqueeze(1), cols.unsqueeze(0)] = seg_lp
            glen[rows] = st.gen_len[:n]
            still = ~st.done[:n]
            step_done += k
            rows = rows[still]
        return tokens_all, lps_all, glen

    def _state(self, nb: int, max_new: int, sampling_key: tuple = ()) -> _DecodeState:
        """Decode buffers + graph for one batch bucket.  Sampling parameters are
        baked into a captured graph, so they are part of the cache key."""
        key = (nb,) + tuple(sampling_key)
        st = self._states.get(key)
        if st is None or st.out_tokens.shape[1] < max_new + 1:
            st = _DecodeState(nb, self.max_blocks_per_seq, max_new, self.device)
            self._states[key] = st
        return st

    def _step_body(self, st: _DecodeState, temperature, top_k, top_p, stop):
        """One decode step over the bucket (graph-capturable: no host syncs)."""
        bs = self.block_size
        blk = st.block_tables.gather(1, (st.positions // bs).long().unsqueeze(1)).squeeze(1)
        st.slot.copy_(blk.long() * bs + (st.positions % bs).long())
        st.seq_lens.copy_(st.positions + 1)
        h = self.model.forward_decode(st.tokens, st.positions, self.kv, st.block_tables, st.seq_lens, st.slot,
                                      self.max_model_len)
        logits = self.model.logits_infer(h)
        from rl_b200.ops.sampling import sample_tokens_graphable

        sample_tokens_graphable(logits, temperature if temperature > 0 else 1.0,
                                1 if temperature == 0 else top_k, top_p, self.seed,
                                st.rng_offset, st.next_tokens, st.next_logprobs)
        if temperature == 0:
            st.next_logprobs.zero_()
        active = ~st.done
        st.out_tokens.scatter_(1, st.step.expand(st.B).unsqueeze(1), st.next_tokens.unsqueeze(1))
        st.out_logprobs.scatter_(1, st.step.expand(st.B).unsqueeze(1), st.next_logprobs.unsqueeze(1))
        st.gen_len.add_(active.to(torch.int32))
        newly = torch.isin(st.next_tokens, stop) | (st.gen_len >= st.max_new)
        st.done.logical_or_(newly)
        st.tokens.copy_(st.next_tokens)
        st.positions.add_(1)
        st.step.add_(1)
        st.rng_offset.add_(1)

    def _capture(self, st: _DecodeState, temperature, top_k, top_p, stop):
        # warm up on a side stream (allocations for the graph pool), then capture
        saved = [t.clone() for t in (st.tokens, st.positions, st.done, st.gen_len, st.step, st.rng_offset,
                                      st.out_tokens, st.out_logprobs)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step_body(st, temperature, top_k, top_p, stop)
        torch.cuda.current_stream().wait_stream(s)
        for t, v in zip((st.tokens, st.positions, st.done, st.gen_len, st.step, st.rng_offset, st.out_tokens,
                         st.out_logprobs), saved):
            t.copy_(v)
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        c0 = launch_count()
        with torch.cuda.graph(g, pool=self._graph_pool, capture_error_mode=self.capture_error_mode):
            self._step_body(st, temperature, top_k, top_p, stop)
        st.native_launches = launch_count() - c0
        add_launches(-st.native_launches)  # captured, not executed
        st.graph = g

    def _decode_eager(self, tokens_all, lps_all, glen, tok0, lengths, block_tables, max_new, temperature, top_k,
                      top_p, stop, gen, done):
        dev = self.device
        bs = self.block_size
        tokens = tok0.clone()
        positions = lengths.to(torch.int32).clone()
        for step in range(1, max_new):
            if bool(done.all()):
                break
            blk = block_tables.gather(1, (positions // bs).long().unsqueeze(1)).squeeze(1)
            slot = blk.long() * bs + (positions % bs).long()
            h = self.model.forward_decode(tokens, positions, self.kv, block_tables, positions + 1, slot,
                                          self.max_model_len)
            if self._route_steps is not None:
                self._route_steps.append(self._take_routes())
            logits = self.model.logits_infer(h)
            if self._topk_steps is not None:
                self._topk_steps.append(self._sampler_topk(logits, temperature, int(self.record_sampler_topk)))
            nt, nlp = sample_tokens(logits, temperature if temperature > 0 else 1.0,
                                    1 if temperature == 0 else top_k, top_p,
                                    seed=self.seed, offset=self.calls * (1 << 24) + step + 1, generator=gen)
            if temperature == 0:
                nlp = torch.zeros_like(nlp)
            active = ~done
            tokens_all[:, step] = torch.where(active, nt, tokens_all[:, step])
            lps_all[:, step] = torch.where(active, nlp, lps_all[:, step])
            glen += active.to(torch.int32)
            done = done | torch.isin(nt, stop) | (glen >= max_new)
            tokens = nt
            positions = positions + 1
        return tokens_all, lps_all, glen
