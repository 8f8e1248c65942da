"""Cross-tokenizer off-policy distillation: offset alignment, vocabulary
projection and the P-KL / gold-loss objectives on tiny models with different
tokenizers (character-level student, two-character teacher)."""

import torch

from rl_b200.algorithms.x_token import (CrossTokenizerDistillationLossFn, VocabProjection, align_by_offsets,
                                        build_xtoken_batch, xtoken_off_policy_distillation_train)

ALPHA = "abcdefgh "


class CharTok:
    """One token per character; id 0 is BOS (empty span)."""

    def vocab(self):
        return ["<s>"] + list(ALPHA)

    def encode(self, text):
        return [0] + [1 + ALPHA.index(c) for c in text], [(0, 0)] + [(i, i + 1) for i in range(len(text))]


class PairTok:
    """Greedy two-character tokens (then single characters); id 0 is BOS."""

    def __init__(self):
        self.v = ["<s>"] + [a + b for a in ALPHA for b in ALPHA] + list(ALPHA)
        self.idx = {s: i for i, s in enumerate(self.v)}

    def vocab(self):
        return self.v

    def encode(self, text):
        ids, offs, i = [0], [(0, 0)], 0
        while i < len(text):
            L = 2 if i + 1 < len(text) and text[i:i + 2] in self.idx and text[i + 1] != " " else 1
            ids.append(self.idx[text[i:i + L]])
            offs.append((i, i + L))
            i += L
        return ids, offs


def test_alignment_and_projection():
    s, t = CharTok(), PairTok()
    _, so = s.encode("abc def")
    _, to = t.encode("abc def")
    ch = align_by_offsets(so, to)
    # teacher: "ab" "c" " d" "ef" -> chunks (a,b)|ab, c|c, (' ',d)|' d', (e,f)|ef
    assert [(c.s0, c.s1, c.t0, c.t1) for c in ch] == [(1, 3, 1, 2), (3, 4, 2, 3), (4, 6, 3, 4), (6, 8, 4, 5)]
    assert [c.exact for c in ch] == [False, True, False, False]
    proj = VocabProjection.from_vocabs(s.vocab(), t.vocab())
    cs, ct = proj.exact_map(1.0)
    # every single character exists in the teacher vocabulary
    assert len(cs) == len(ALPHA) + 1
    p = torch.zeros(1, len(s.vocab()))
    p[0, 1 + ALPHA.index("c")] = 1.0
    q = proj.project(p)
    assert q[0, t.idx["c"]] == 1.0 and q.sum() == 1.0


def _teacher():
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM

    cfg = ModelConfig(name="teacher", vocab_size=128, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=16, ffn_hidden_size=128, rope_theta=10000.0, max_position_embeddings=256)
    m = TransformerLM(cfg, dtype=torch.float32, seed=11)

    @torch.no_grad()
    def topk(ids, lengths, k=8):
        B, T = ids.shape
        outs_i, outs_l = torch.zeros(B, T, k, dtype=torch.long), torch.zeros(B, T, k)
        for b in range(B):
            L = int(lengths[b])
            pos = torch.arange(L, dtype=torch.int32)
            h = m(ids[b, :L], pos, torch.tensor([0, L], dtype=torch.int32), L)
            lp = torch.log_softmax(m.logits(h).float(), -1)
            v, i = lp.topk(k, -1)
            outs_i[b, :L], outs_l[b, :L] = i, v
        return outs_i, outs_l

    return topk


def test_xtoken_distillation_reduces_kd():
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker

    s, t = CharTok(), PairTok()
    teacher = _teacher()
    texts = ["abc def gh", "head bag", "fed cab", "ache deaf", "bead fade", "cafe bed", "hag dab", "gab had"]
    scfg = ModelConfig(name="student", vocab_size=16, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                       head_dim=16, ffn_hidden_size=128, rope_theta=10000.0, max_position_embeddings=256)
    for gold, xt in ((False, False), (True, False), (True, True)):
        pc = {"max_total_sequence_length": 64, "precision": "float32", "train_global_batch_size": 8,
              "optimizer": {"kwargs": {"lr": 3e-3, "weight_decay": 0.0}},
              "generation": {"temperature": 1.0, "max_new_tokens": 4},
              "sequence_packing": {"train_mb_tokens": 128, "logprob_mb_tokens": 128}}
        student = PolicyWorker(pc, model_cfg=scfg, seed=2)
        cfg = {"gold_loss": gold, "xtoken_loss": xt, "temperature": 1.0, "kl_loss_weight": 1.0,
               "ce_loss_scale": 0.0, "uncommon_topk": 16}
        b = build_xtoken_batch(texts, s, t, teacher)
        assert b["xt_valid"].sum() > 0 and b["teacher_topk_ids"].shape[-1] == 8
        res = xtoken_off_policy_distillation_train(student, teacher, texts, s, t, cfg, batch_size=8, max_steps=8,
                                                   teacher_vocab_size=128)
        kl = [r["kl_loss"] for r in res]
        assert kl[-1] < kl[0], (gold, xt, kl)
