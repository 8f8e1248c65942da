"""Eagle3 draft head for speculative decoding, trained online on the policy's
own hidden states.

Reference: the Eagle3 drafter the reference attaches to its policy worker
(``policy.draft``: ``enabled``, ``speculator_type: eagle3``, ``loss_weight``,
``nemo_rl/models/policy/draft_config.py:64``, ``models/megatron/draft/*``) and the
alignment documented in its Eagle3 guide: the draft at position ``t`` sees the
policy's hidden features of position ``t`` and the embedding of token ``t + 1``
and predicts token ``t + 2``.

The head here:

* features: the residual stream after three policy layers (early / middle /
  late; ``aux_layers``), concatenated ``[T, 3H]`` and fused by ``fc`` to ``[T, H]``;
* input: ``in_proj([rmsnorm(embedding of the next token); rmsnorm(feature)])``
  (``2H -> H``), the policy's own (detached) token embedding;
* one decoder layer with its own attention and MLP, a final norm and its own
  LM head (initialised from the policy's output layer), built as a one-layer
  ``TransformerLM`` fed ``hidden_in`` (its tied embedding table IS the head);
* training: cross-entropy of the token two positions ahead (the token the
  policy actually sampled, an unbiased sample of the policy distribution the
  reference distils), plus ``ttt_steps - 1`` extra unrolled steps in which the
  draft's own output hidden replaces the policy feature, which is what it
  consumes when it proposes several tokens in a row;
* decoding (``RolloutEngine``): prefill over the prompt with the policy's
  prefill features, proposals feeding back the draft's hidden, and after each
  verification the draft's cache entries of the accepted positions rewritten
  from the policy's verified features.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from rl_b200.ops.linear import linear
from rl_b200.ops.norm import rms_norm

__all__ = ["Eagle3Draft", "default_aux_layers", "shift_features"]


def default_aux_layers(num_layers: int) -> tuple:
    """Early / middle / late feature layers of an ``num_layers``-deep policy."""
    cand = (1, num_layers // 2 - 1, num_layers - 4)
    return tuple(sorted({min(max(0, c), num_layers - 1) for c in cand})) if num_layers >= 3 else \
        tuple(range(num_layers))


def shift_features(feats: torch.Tensor, cu_seqlens: torch.Tensor) -> torch.Tensor:
    """Per packed sequence, features of position ``t - 1`` at position ``t``
    (zeros at each sequence's first position)."""
    out = torch.zeros_like(feats)
    out[1:] = feats[:-1]
    starts = cu_seqlens[:-1].long()
    out[starts] = 0
    return out


class Eagle3Draft(nn.Module):
    def __init__(self, target, aux_layers: Optional[tuple] = None, seed: int = 0, ttt_steps: int = 2):
        super().__init__()
        from rl_b200.models.transformer import TransformerLM

        if target.ps.tp_size > 1 or target.ps.pp_size > 1:
            raise NotImplementedError("the Eagle3 draft runs unsharded (policy TP = PP = 1)")
        c = target.cfg
        H = c.hidden_size
        n_feat = len(aux_layers or default_aux_layers(c.num_layers))
        self.aux_layers = tuple(aux_layers or default_aux_layers(c.num_layers))
        self.ttt_steps = max(1, int(ttt_steps))
        dcfg = c.replace(num_layers=1, tie_word_embeddings=True)
        # one decoder layer + final norm; the tied table serves as the draft's LM head
        self.body = TransformerLM(dcfg, target.ps, device=target.device, dtype=target.dtype, seed=seed + 7717)
        with torch.no_grad():
            self.body.param("model.embed_tokens.weight").copy_(target.lm_head_weight())
        dev, dt = target.device, target.dtype
        g = torch.Generator(device=dev).manual_seed(seed + 31)
        self.fc = nn.Parameter((torch.randn(H, n_feat * H, generator=g, device=dev) * (n_feat * H) ** -0.5).to(dt))
        self.in_proj = nn.Parameter((torch.randn(H, 2 * H, generator=g, device=dev) * (2 * H) ** -0.5).to(dt))
        self.norm_emb = nn.Parameter(torch.ones(H, device=dev, dtype=dt))
        self.norm_feat = nn.Parameter(torch.ones(H, device=dev, dtype=dt))
        self.eps = c.rms_eps

    # engine-facing attributes of the draft's single layer
    @property
    def cfg(self):
        return self.body.cfg

    @property
    def nkv(self) -> int:
        return self.body.nkv

    @property
    def hd(self) -> int:
        return self.body.hd

    @property
    def ps(self):
        return self.body.ps

    def fuse(self, feats: torch.Tensor) -> torch.Tensor:
        """``[T, n_feat * H]`` policy features -> ``[T, H]``."""
        return linear(feats, self.fc)

    def combine(self, emb: torch.Tensor, feat_h: torch.Tensor) -> torch.Tensor:
        """Draft layer input from the next token's embedding and an H-wide feature."""
        z = torch.cat([rms_norm(emb, self.norm_emb, self.eps), rms_norm(feat_h, self.norm_feat, self.eps)], -1)
        return linear(z, self.in_proj)

    def logits_infer(self, h: torch.Tensor) -> torch.Tensor:
        return self.body.logits_infer(h)

    # ------------------------------------------------------------- training
    def train_loss(self, emb_next: torch.Tensor, feats: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor,
                   positions: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
        """Mean cross-entropy over ``mask`` and the unrolled steps.  Row ``t`` holds
        the policy features of position ``t`` (``feats``), the embedding of token
        ``t + 1`` (``emb_next``) and the label token ``t + 2`` (``targets``); step
        ``s`` >= 1 feeds the draft's own hidden of row ``t - 1`` as the feature
        and predicts ``s`` positions further."""
        from rl_b200.ops.fused_linear_logprob import linear_logprobs

        feat_h = self.fuse(feats)
        losses = []
        cur_mask = mask
        emb, tgt = emb_next, targets
        for s in range(self.ttt_steps):
            h = self.body(torch.zeros_like(targets), positions, cu_seqlens, max_seqlen,
                          hidden_in=self.combine(emb, feat_h))
            lp, _ = linear_logprobs(h, self.body.lm_head_weight(), tgt)
            m = cur_mask.to(lp.dtype)
            losses.append(-(lp * m).sum() / m.sum().clamp_min(1))
            if s + 1 < self.ttt_steps:
                # next step: row t takes the draft's hidden of row t - 1 and looks one token further
                feat_h = shift_features(h, cu_seqlens)
                emb = torch.roll(emb, -1, 0)
                tgt = torch.roll(tgt, -1, 0)
                shifted = torch.roll(cur_mask, -1, 0)
                last = cu_seqlens[1:].long() - 1
                shifted[last] = False
                cur_mask = cur_mask & shifted
        return torch.stack(losses).mean()

    # ------------------------------------------------------------- decoding
    def prefill(self, emb: torch.Tensor, feats_prev: torch.Tensor, positions, cu_seqlens, max_seqlen, kv,
                slot_mapping, last_token_index) -> torch.Tensor:
        """Cache the draft layer's K/V over the prompt: row ``t`` gets the policy
        features of ``t - 1`` (``feats_prev``, zeros at sequence starts) and the
        embedding of token ``t``."""
        z = self.combine(emb, self.fuse(feats_prev))
        return self.body.forward_prefill(None, positions, cu_seqlens, max_seqlen, kv, slot_mapping,
                                         last_token_index, hidden_in=z)

    @torch.no_grad()
    def step(self, emb: torch.Tensor, feat_h: torch.Tensor, positions, kv, block_tables, seq_lens, slot_mapping,
             max_seq_len: int) -> torch.Tensor:
        """One draft position per row: returns the draft hidden ``[B, H]`` (its
        logits come from ``logits_infer``; it is also the next step's feature)."""
        z = self.combine(emb, feat_h)
        return self.body.forward_decode(positions, positions, kv, block_tables, seq_lens, slot_mapping, max_seq_len,
                                        hidden_in=z)


class DFlashDraft(Eagle3Draft):
    """Block drafter: ``block_size`` tokens proposed in ONE forward pass.

    Reference: the ``dflash`` speculator type of the reference's draft heads
    (``nemo_rl/models/generation/vllm/speculator_runtime.py:23``; its drafts carry a
    ``mask_embedding`` parameter, ``vllm/draft_utils.py:112``).  Here the block
    of a position ``t`` is a short sequence of its own: row 0 holds
    ``combine(embedding of token t + 1, fused feature of t)``, rows 1..k-1 hold
    ``combine(mask embedding, fused feature of t)``; rows attend causally within
    the block (block-local positions 0..k-1) and row j predicts token
    ``t + 2 + j``.  The target's multi-layer features of ``t`` are the only
    context, so training on sampled anchor positions and proposing at decode time
    see the same computation, and drafting needs no draft KV cache."""

    def __init__(self, target, aux_layers: Optional[tuple] = None, seed: int = 0, block_size: int = 4):
        super().__init__(target, aux_layers=aux_layers, seed=seed, ttt_steps=1)
        self.block_size = max(1, int(block_size))
        H = target.cfg.hidden_size
        g = torch.Generator(device=target.device).manual_seed(seed + 97)
        self.mask_embedding = nn.Parameter((torch.randn(H, generator=g, device=target.device) * 0.02)
                                           .to(target.dtype))

    def _block_inputs(self, emb_first: torch.Tensor, feat_h: torch.Tensor, k: int) -> torch.Tensor:
        """[n, H] first-row embeddings and features -> [n * k, H] block inputs."""
        n, H = emb_first.shape
        emb = self.mask_embedding.view(1, 1, H).expand(n, k, H).clone()
        emb[:, 0] = emb_first
        feat = feat_h.unsqueeze(1).expand(n, k, H)
        return self.combine(emb.reshape(n * k, H), feat.reshape(n * k, H))

    def _block_forward(self, z: torch.Tensor, n: int, k: int) -> torch.Tensor:
        dev = z.device
        pos = torch.arange(k, device=dev, dtype=torch.int32).repeat(n)
        cu = torch.arange(0, n * k + 1, k, device=dev, dtype=torch.int32)
        return self.body(torch.zeros(n * k, dtype=torch.long, device=dev), pos, cu, k, hidden_in=z)

    def train_loss(self, emb_next: torch.Tensor, feats: torch.Tensor, tokens: torch.Tensor,
                   cu_seqlens: torch.Tensor, max_anchors: int = 1024, seed: int = 0) -> torch.Tensor:
        """Cross-entropy over sampled anchor positions ``t`` (row ``t`` of
        ``emb_next`` is the embedding of token ``t + 1``, of ``feats`` the policy
        features of ``t``; ``tokens`` the packed ids): each anchor's block predicts
        tokens ``t + 2 .. t + 1 + k`` (rows past its sequence's end are masked)."""
        from rl_b200.ops.fused_linear_logprob import linear_logprobs

        k = self.block_size
        T = tokens.numel()
        dev = tokens.device
        seq_end = torch.repeat_interleave(cu_seqlens[1:].long(), (cu_seqlens[1:] - cu_seqlens[:-1]).long())
        idx = torch.arange(T, device=dev)
        valid = idx + 2 < seq_end
        anchors = idx[valid]
        if anchors.numel() == 0:
            return feats.sum() * 0.0
        if anchors.numel() > max_anchors:
            g = torch.Generator(device="cpu").manual_seed(seed)
            anchors = anchors[torch.randperm(anchors.numel(), generator=g)[:max_anchors].to(dev)]
        n = anchors.numel()
        z = self._block_inputs(emb_next[anchors], self.fuse(feats[anchors]), k)
        h = self._block_forward(z, n, k)
        tpos = anchors.unsqueeze(1) + 2 + torch.arange(k, device=dev).unsqueeze(0)      # [n, k]
        ok = tpos < seq_end[anchors].unsqueeze(1)
        tgt = tokens[tpos.clamp(max=T - 1)].reshape(-1)
        lp, _ = linear_logprobs(h, self.body.lm_head_weight(), tgt)
        m = ok.reshape(-1).to(lp.dtype)
        return -(lp * m).sum() / m.sum().clamp_min(1)

    @torch.no_grad()
    def propose(self, emb_last: torch.Tensor, feat_h: torch.Tensor, k: Optional[int] = None) -> torch.Tensor:
        """One forward for every sequence's block: returns ``[B * k, V]`` logits
        (row j of sequence b proposes the token ``j + 1`` places after ``last``)."""
        k = k or self.block_size
        B = emb_last.shape[0]
        h = self._block_forward(self._block_inputs(emb_last, feat_h, k), B, k)
        return self.logits_infer(h)
