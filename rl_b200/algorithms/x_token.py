"""Cross-tokenizer (x-token) off-policy distillation.

A student and a teacher with DIFFERENT tokenizers read the same text.

* Alignment (``align_by_offsets``): both tokenizations carry the character span
  of every token; walking both sequences by character END position pairs
  student token runs with teacher token runs that cover exactly the same
  characters (a chunk).  A chunk is *exact* when it is one token on each side.
* Projection (``VocabProjection``): a sparse ``[V_s, V_t]`` map from student to
  teacher tokens - built from the token strings (identical strings map with
  likelihood 1; otherwise the student string's first teacher piece by longest
  match) or loaded from the reference's top-k file format
  (``{"indices": [V_s, k], "likelihoods": [V_s, k]}``).
* Loss (``CrossTokenizerDistillationLossFn``) at the first token of every
  aligned chunk, where both models predict the start of the same character span:
    - P-KL (``gold_loss: false``): KL(teacher || student projected through the map)
      over the teacher's top-k ids, renormalised;
    - gold loss (``gold_loss: true``): KL on the *common* vocabulary (student ids
      with an exact map; ``xtoken_loss: true`` relaxes "exact" to a map weight of
      at least 0.6) plus the L1 distance between the sorted probability tails of
      the *uncommon* ids (top ``uncommon_topk``), times ``T^2``;
  combined with the student's next-token cross-entropy as
  ``kl_loss_weight * kd + ce_loss_scale * ce`` (or, with
  ``dynamic_loss_scaling``, the KD term rescaled to the detached CE magnitude).

Reference: ``nemo_rl/algorithms/xtoken_off_policy_distillation.py`` (loop,
``:622``), ``nemo_rl/algorithms/x_token/token_aligner.py`` (offset alignment,
``align_by_offsets_cluster`` ``:1551``) and ``CrossTokenizerDistillationLossFn``
(``nemo_rl/algorithms/loss/loss_functions.py:2379``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Protocol

import torch

from rl_b200.algorithms.loss.interfaces import LossInputType, LossType
from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["align_by_offsets", "Chunk", "VocabProjection", "CrossTokenizerDistillationLossFn",
           "build_xtoken_batch", "xtoken_off_policy_distillation_train", "OffsetTokenizer"]


class OffsetTokenizer(Protocol):
    """``encode(text) -> (ids, [(char_start, char_end), ...])`` and ``vocab() -> list[str]``."""

    def encode(self, text: str) -> tuple[list[int], list[tuple[int, int]]]: ...

    def vocab(self) -> list[str]: ...


@dataclass
class Chunk:
    s0: int
    s1: int  # student tokens [s0, s1)
    t0: int
    t1: int  # teacher tokens [t0, t1)

    @property
    def exact(self) -> bool:
        return self.s1 - self.s0 == 1 and self.t1 - self.t0 == 1


def align_by_offsets(s_off: list, t_off: list) -> list[Chunk]:
    """Pair student / teacher token runs covering the same characters.  Tokens
    with an empty span (special tokens) are skipped; a run ends where both
    sides reach the same character end with the same start."""
    def content(offs):
        return [i for i, (a, b) in enumerate(offs) if b > a]

    si, ti = content(s_off), content(t_off)
    out: list[Chunk] = []
    i = j = 0
    while i < len(si) and j < len(ti):
        s_start, t_start = s_off[si[i]][0], t_off[ti[j]][0]
        i0, j0 = i, j
        s_end, t_end = s_off[si[i]][1], t_off[ti[j]][1]
        while s_end != t_end:
            if s_end < t_end:
                i += 1
                if i >= len(si):
                    return out
                s_end = s_off[si[i]][1]
            else:
                j += 1
                if j >= len(ti):
                    return out
                t_end = t_off[ti[j]][1]
        # contiguous runs only (no skipped specials inside)
        if s_start == t_start and si[i] - si[i0] == i - i0 and ti[j] - ti[j0] == j - j0:
            out.append(Chunk(si[i0], si[i] + 1, ti[j0], ti[j] + 1))
        i += 1
        j += 1
    return out


class VocabProjection:
    """Sparse student -> teacher token map ``M [V_s, V_t]`` (rows sum to <= 1)."""

    def __init__(self, indices: torch.Tensor, likelihoods: torch.Tensor, v_teacher: int):
        self.indices, self.likelihoods = indices.long(), likelihoods.float()
        self.v_s, self.v_t = indices.shape[0], v_teacher
        rows = torch.arange(self.v_s).repeat_interleave(indices.shape[1])
        keep = self.likelihoods.reshape(-1) > 0
        self.M = torch.sparse_coo_tensor(torch.stack([rows[keep], self.indices.reshape(-1)[keep]]),
                                         self.likelihoods.reshape(-1)[keep], (self.v_s, self.v_t),
                                         check_invariants=True).coalesce()
        top_w, top_i = self.likelihoods.max(-1)
        self.best_teacher = self.indices.gather(1, top_i.unsqueeze(1)).squeeze(1)
        self.best_weight = top_w

    @staticmethod
    def load(path: str, v_teacher: int) -> "VocabProjection":
        d = torch.load(path, map_location="cpu")
        return VocabProjection(d["indices"], d["likelihoods"], v_teacher)

    @staticmethod
    def from_vocabs(student_vocab: list[str], teacher_vocab: list[str], v_student: Optional[int] = None,
                    v_teacher: Optional[int] = None) -> "VocabProjection":
        """``v_student`` / ``v_teacher``: the models' logit widths when they exceed
        the tokenizers' vocabularies (padded embedding tables); extra ids map to nothing."""
        t_index = {s: i for i, s in enumerate(teacher_vocab)}
        max_len = max((len(s) for s in teacher_vocab), default=1)
        vs = max(len(student_vocab), v_student or 0)
        idx = torch.zeros(vs, 1, dtype=torch.long)
        lik = torch.zeros(vs, 1)
        for i, s in enumerate(student_vocab):
            if s in t_index:
                idx[i, 0], lik[i, 0] = t_index[s], 1.0
                continue
            for L in range(min(len(s), max_len), 0, -1):  # first teacher piece, longest match
                if s[:L] in t_index:
                    idx[i, 0], lik[i, 0] = t_index[s[:L]], 0.5
                    break
        return VocabProjection(idx, lik, max(len(teacher_vocab), v_teacher or 0))

    def project(self, probs: torch.Tensor) -> torch.Tensor:
        """Student probabilities ``[N, V_s]`` -> teacher-vocabulary mass ``[N, V_t]`` (fp32)."""
        p = probs.float()
        if p.shape[1] != self.v_s:  # logits wider / narrower than the map: unmapped ids carry no mass
            p = torch.nn.functional.pad(p, (0, self.v_s - p.shape[1])) if p.shape[1] < self.v_s else p[:, :self.v_s]
        return torch.sparse.mm(self.M.to(probs.device).t(), p.t()).t()

    def exact_map(self, threshold: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
        """(student ids, teacher ids) of the common vocabulary: students whose
        best teacher map has weight >= threshold, one student per teacher id."""
        ok = self.best_weight >= threshold
        s = torch.nonzero(ok).flatten()
        t = self.best_teacher[s]
        # collisions: keep the first student id per teacher id
        seen, keep = set(), []
        for a, b in zip(s.tolist(), t.tolist()):
            if b not in seen:
                seen.add(b)
                keep.append(a)
        s = torch.tensor(keep, dtype=torch.long)
        return s, self.best_teacher[s]


class CrossTokenizerDistillationLossFn:
    """See the module docstring.  Consumes full student logits (``LOGIT``
    input) and per-sample data ``xt_s_pos / xt_t_pos / xt_valid`` (aligned
    chunk starts, ``[B, C]``) plus the teacher's top-k next-token log-probs
    ``teacher_topk_ids / teacher_topk_logprobs`` (``[B, T_t, k]``)."""

    loss_type = LossType.TOKEN_LEVEL
    input_type = LossInputType.LOGIT

    def __init__(self, cfg: dict, projection: VocabProjection):
        self.gold = bool(cfg.get("gold_loss", False))
        self.xtoken = bool(cfg.get("xtoken_loss", False))
        if self.xtoken and not self.gold:
            raise ValueError("xtoken_loss is a modifier of gold_loss")
        self.T = float(cfg.get("temperature", 1.0))
        self.uncommon_topk = int(cfg.get("uncommon_topk", 8192))
        self.reverse = bool(cfg.get("reverse_kl", False))
        self.exact_only = bool(cfg.get("exact_token_match_only", False))
        self.kl_w = float(cfg.get("kl_loss_weight", 1.0))
        self.ce_w = float(cfg.get("ce_loss_scale", 1.0))
        self.dynamic = bool(cfg.get("dynamic_loss_scaling", False))
        self.proj = projection
        if self.gold:
            self.common_s, self.common_t = projection.exact_map(0.6 if self.xtoken else 1.0)

    def _kd(self, s_logits: torch.Tensor, t_ids: torch.Tensor, t_lp: torch.Tensor) -> torch.Tensor:
        """Per-chunk distillation term: student logits ``[C, V_s]``, teacher
        top-k ``[C, k]`` ids / log-probs."""
        T = self.T
        ps = torch.softmax(s_logits.float() / T, -1)
        pt_k = torch.softmax(t_lp.float() / T, -1)           # teacher top-k, renormalised
        if not self.gold:
            q = self.proj.project(ps).gather(1, t_ids.long()).clamp_min(1e-12)
            q = q / q.sum(-1, keepdim=True)
            if self.reverse:
                return (q * (q.log() - pt_k.clamp_min(1e-12).log())).sum(-1)
            return (pt_k * (pt_k.clamp_min(1e-12).log() - q.log())).sum(-1)
        # gold loss: dense teacher distribution over its top-k ids
        C = s_logits.shape[0]
        pt = torch.zeros(C, self.proj.v_t, device=s_logits.device).scatter_(1, t_ids.long(), pt_k)
        cs, ct = self.common_s.to(s_logits.device), self.common_t.to(s_logits.device)
        ps_c, pt_c = ps[:, cs], pt[:, ct]
        kl = (pt_c * (pt_c.clamp_min(1e-12).log() - ps_c.clamp_min(1e-12).log())).sum(-1)
        s_unc = ps.clone()
        s_unc[:, cs] = 0
        t_unc = pt.clone()
        t_unc[:, ct] = 0
        k = min(self.uncommon_topk, s_unc.shape[1], t_unc.shape[1])
        l1 = (s_unc.topk(k, -1)[0] - t_unc.topk(k, -1)[0]).abs().sum(-1)
        return (kl + l1) * T * T

    def __call__(self, logits: torch.Tensor, data: BatchedDataDict, global_valid_seqs, global_valid_toks):
        # logits [n, W-1, V_s]: position j predicts token j+1
        n = logits.shape[0]
        mask = data["token_mask"][:, 1:logits.shape[1] + 1].float() * data["sample_mask"].float().unsqueeze(-1)
        tgt = data["input_ids"][:, 1:logits.shape[1] + 1].long()
        lp = torch.log_softmax(logits.float(), -1)
        tok_lp = lp.gather(-1, tgt.unsqueeze(-1)).squeeze(-1)
        ce = -(tok_lp * mask).sum() / global_valid_toks.clamp_min(1)
        # chunk starts: student predicts token s0 at position s0-1, teacher t0 at t0-1
        s_pos = data["xt_s_pos"].long() - 1
        t_pos = data["xt_t_pos"].long() - 1
        valid = data["xt_valid"].bool() & (s_pos >= 0) & (t_pos >= 0) & (s_pos < logits.shape[1])
        if self.exact_only:
            valid = valid & data["xt_exact"].bool()
        b, c = torch.nonzero(valid, as_tuple=True)
        if b.numel() > 0:
            s_log = logits[b, s_pos[b, c]]
            t_ids = data["teacher_topk_ids"][b, t_pos[b, c]]
            t_lp = data["teacher_topk_logprobs"][b, t_pos[b, c]]
            # token-level normalisation (global valid tokens), like the CE term
            kd = self._kd(s_log, t_ids, t_lp).sum() / global_valid_toks.clamp_min(1)
        else:
            kd = logits.sum() * 0.0
        if self.dynamic:
            scale = (ce.detach() / kd.detach().clamp_min(1e-8)) if b.numel() > 0 else torch.zeros(())
            loss = kd * scale + ce
        else:
            scale = torch.tensor(self.kl_w)
            loss = self.kl_w * kd + self.ce_w * ce
        acc = ((lp.argmax(-1) == tgt).float() * mask).sum() / global_valid_toks.clamp_min(1)
        metrics = {"loss": loss.detach(), "kl_loss": kd.detach(), "ce_loss": ce.detach(),
                   "kl_loss_scale_max": torch.as_tensor(scale).detach().float(), "accuracy": acc.detach(),
                   "num_valid_samples": torch.tensor(float(n))}
        return loss, metrics


def build_xtoken_batch(texts: list[str], s_tok: OffsetTokenizer, t_tok: OffsetTokenizer,
                       teacher_topk: Callable[[torch.Tensor, torch.Tensor], tuple[torch.Tensor, torch.Tensor]],
                       max_len: int = 512) -> BatchedDataDict:
    """Tokenise ``texts`` with both tokenizers, align them, run the teacher
    (``teacher_topk(ids [B, T_t], lengths) -> (ids, log-probs) [B, T_t, k]``) and
    pack the student's training batch."""
    s_enc = [s_tok.encode(t) for t in texts]
    t_enc = [t_tok.encode(t) for t in texts]
    B = len(texts)
    Ls = [min(len(e[0]), max_len) for e in s_enc]
    Lt = [min(len(e[0]), max_len) for e in t_enc]
    S, Tt = max(Ls), max(Lt)
    ids = torch.zeros(B, S, dtype=torch.long)
    tids = torch.zeros(B, Tt, dtype=torch.long)
    chunks = []
    for b in range(B):
        ids[b, :Ls[b]] = torch.tensor(s_enc[b][0][:Ls[b]])
        tids[b, :Lt[b]] = torch.tensor(t_enc[b][0][:Lt[b]])
        ch = [c for c in align_by_offsets(s_enc[b][1][:Ls[b]], t_enc[b][1][:Lt[b]])]
        chunks.append(ch)
    C = max(1, max(len(c) for c in chunks))
    s_pos = torch.zeros(B, C, dtype=torch.long)
    t_pos = torch.zeros(B, C, dtype=torch.long)
    ok = torch.zeros(B, C, dtype=torch.bool)
    ex = torch.zeros(B, C, dtype=torch.bool)
    for b, ch in enumerate(chunks):
        for c, k in enumerate(ch):
            s_pos[b, c], t_pos[b, c], ok[b, c], ex[b, c] = k.s0, k.t0, True, k.exact
    top_ids, top_lp = teacher_topk(tids, torch.tensor(Lt))
    tm = torch.zeros(B, S)
    for b in range(B):
        tm[b, 1:Ls[b]] = 1
    return BatchedDataDict({"input_ids": ids, "input_lengths": torch.tensor(Ls), "token_mask": tm,
                            "sample_mask": torch.ones(B), "xt_s_pos": s_pos, "xt_t_pos": t_pos, "xt_valid": ok,
                            "xt_exact": ex, "teacher_topk_ids": top_ids, "teacher_topk_logprobs": top_lp})


def xtoken_off_policy_distillation_train(student, teacher_topk, texts: list[str], s_tok: OffsetTokenizer,
                                         t_tok: OffsetTokenizer, loss_cfg: dict,
                                         projection: Optional[VocabProjection] = None, batch_size: int = 8,
                                         max_steps: int = 1, max_len: int = 512, teacher_vocab_size: int = 0,
                                         logger=None) -> list[dict]:
    """Off-policy cross-tokenizer distillation: each step packs ``batch_size``
    texts, scores them with the teacher and takes one student optimizer step.
    ``teacher_vocab_size``: the teacher model's logit width (if above its
    tokenizer's vocabulary)."""
    proj = projection or VocabProjection.from_vocabs(s_tok.vocab(), t_tok.vocab(),
                                                     student.model_cfg.vocab_size, teacher_vocab_size)
    loss_fn = CrossTokenizerDistillationLossFn(loss_cfg, proj)
    out = []
    for step in range(max_steps):
        chunk = [texts[(step * batch_size + i) % len(texts)] for i in range(batch_size)]
        batch = build_xtoken_batch(chunk, s_tok, t_tok, teacher_topk, max_len)
        res = student.train(batch, loss_fn, gbs=batch_size)
        out.append(res)
        if logger is not None:
            logger.log_metrics({f"train/{k}": v for k, v in res.items() if isinstance(v, (int, float))}, step)
    return out
