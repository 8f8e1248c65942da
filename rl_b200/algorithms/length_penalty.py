"""Per-prompt-group length bonuses and penalties on rollout rewards
(``grpo.length_penalty``).

Every adjustment is resolved inside one prompt group (``group_size``
contiguous rollouts of the same prompt) and, unless stated otherwise, only
rollouts with ``reward > 0`` take part.  Lengths are measured on three
channels: ``reasoning`` (the model's thinking), ``answer`` (its visible
output) and ``total`` (their sum), in ``length_type`` units: ``tokens``
(re-tokenised text, characters when no tokenizer is given), ``chars``, or
``all_generated_tokens`` (every token of the assistant turns; total only).

Additive adjustments (summed, the result clamped at 0 so a correct rollout
can lose its reward but never turns negative):

* ``<channel>_bonus``: flat bonus to the shortest non-empty positive rollout,
  when it is a top scorer.
* ``longest_<channel>_penalty``: flat penalty on the longest of the top
  scorers (the best ``top_percentile`` of the positive rewards); needs two.
* ``group_<channel>_length_penalty_coeff``: dense, zero-centred: each
  positive rollout's weight ``1 - (len - min) / (max - min)`` minus the mean
  weight, times the coefficient.  ``group_length_penalty_profile_gate``
  switches the three coefficients off for a group whose mean length does not
  exceed a per-prompt limit ``profile_band[channel][field]``.
* ``<channel>_zmad_threshold`` / ``_penalty``: flat penalty on high-side
  outliers by the Iglewicz-Hoaglin modified z-score
  ``0.6745 (len - median) / MAD`` (none when ``MAD / median < 0.015``).
* profiled length penalty, from per-prompt ``profiled_rewards`` /
  ``profiled_output_lengths`` of a profiling run (passing = reward above
  ``profiled_reward_correct_threshold``; needs
  ``profiled_length_min_samples`` of them): ``constant_over_n_std``
  subtracts ``profiled_length_penalty`` at or past ``mean + n_std * std``
  (not on rollouts the group-relative channels already pushed down);
  ``zero_over_max`` zeroes rollouts longer than the longest passing one.
* ``pass_rate_length_penalty_weight`` ``w``: ``-w * rho * len / l_max`` on
  correct rollouts (``rho`` the group's pass rate, ``l_max`` the longest
  correct total length).

Then ``profile_band_<channel>`` multiplies the rewards of originally correct
rollouts by a per-prompt (or global) band: 1 up to ``a``, linear to ``f`` at
``b``, ``f`` beyond.

Adjustments assume binary (0/1) single-component rewards: a group with a
graded, negative or multi-component reward is left as it is (warned once per
agent), except that ``zero_over_max`` with
``profiled_length_allow_non_binary_rewards`` still caps graded non-negative
groups.  Rows flagged ``low_effort_applied`` skip every adjustment.

Reference: ``nemo_rl/utils/length_penalty.py`` (``apply_group_length_penalties``
``:333``, config ``:56-178``) and its guide ``docs/guides/length-penalty.md``;
the metrics keep the reference's ``length_penalty/*`` names.
"""

from __future__ import annotations

import dataclasses
import logging
import math
import re
import statistics
from typing import Any, Optional

import torch

__all__ = ["LengthPenaltyParams", "LengthPenaltyConfig", "apply_group_length_penalties",
           "split_reasoning_answer", "apply_length_penalty_to_rollout", "CHANNELS"]

log = logging.getLogger(__name__)

CHANNELS = ("reasoning", "answer", "total")
_LENGTH_TYPES = ("tokens", "chars", "all_generated_tokens")
_PROFILED_TYPES = ("constant_over_n_std", "zero_over_max")
_ZMAD_MIN_MAD_REL = 0.015
_BINARY_TOL = 1e-6
_THINK = re.compile(r"<think>(.*?)(?:</think>|$)", re.S)


@dataclasses.dataclass
class LengthPenaltyParams:
    """Settings of one agent (``default`` or an ``agent_overrides`` entry)."""

    enabled: bool = True
    length_type: str = "tokens"
    top_percentile: float = 0.5
    reasoning_bonus: float = 0.0
    answer_bonus: float = 0.0
    total_bonus: float = 0.0
    longest_reasoning_penalty: float = 0.0
    longest_answer_penalty: float = 0.0
    longest_total_penalty: float = 0.0
    group_reasoning_length_penalty_coeff: float = 0.0
    group_answer_length_penalty_coeff: float = 0.0
    group_total_length_penalty_coeff: float = 0.0
    reasoning_zmad_threshold: float = 0.0
    reasoning_zmad_penalty: float = 0.0
    answer_zmad_threshold: float = 0.0
    answer_zmad_penalty: float = 0.0
    total_zmad_threshold: float = 0.0
    total_zmad_penalty: float = 0.0
    profiled_length_penalty: float = 0.0
    profiled_length_penalty_type: str = "constant_over_n_std"
    profiled_length_n_std: float = 1.0
    profiled_length_min_samples: int = 2
    profiled_reward_correct_threshold: float = 0.0
    profiled_length_allow_non_binary_rewards: bool = False
    pass_rate_length_penalty_weight: float = 0.0
    profile_band_total: bool = False
    profile_band_reasoning: bool = False
    profile_band_answer: bool = False
    group_length_penalty_profile_gate: bool = False
    group_length_penalty_profile_gate_channel: str = "total"
    group_length_penalty_profile_gate_field: str = "a"
    group_length_penalty_profile_gate_positive_only: bool = True

    @classmethod
    def keys(cls) -> set[str]:
        return {f.name for f in dataclasses.fields(cls)}

    @classmethod
    def check_keys(cls, d: dict, where: str) -> None:
        """Reject unknown keys and bad enumerations (a misspelt key would
        otherwise leave a penalty silently off)."""
        unknown = set(d) - cls.keys()
        if unknown:
            raise ValueError(f"{where}: unknown length_penalty keys {sorted(unknown)}")
        enums = {"length_type": _LENGTH_TYPES, "profiled_length_penalty_type": _PROFILED_TYPES,
                 "group_length_penalty_profile_gate_channel": CHANNELS,
                 "group_length_penalty_profile_gate_field": ("a", "b", "f")}
        for k, allowed in enums.items():
            if k in d and d[k] not in allowed:
                raise ValueError(f"{where}: {k}={d[k]!r} is not one of {allowed}")


def _check_band_channel(ch: Any, where: str) -> dict:
    if not isinstance(ch, dict) or not {"a", "b"} <= set(ch) or set(ch) - {"a", "b", "f"}:
        raise ValueError(f"{where}: a profile band channel needs keys a, b (and f), got {ch!r}")
    a, b, f = float(ch["a"]), float(ch["b"]), float(ch.get("f", 1.0))
    if b <= a:
        raise ValueError(f"{where}: profile band requires b > a, got a={a}, b={b}")
    if not 0.0 <= f <= 1.0:
        raise ValueError(f"{where}: profile band f must lie in [0, 1], got {f}")
    return {"a": a, "b": b, "f": f}


def _check_resolved(name: str, p: dict) -> None:
    zero_over_max = p["profiled_length_penalty_type"] == "zero_over_max"
    if zero_over_max and p["profiled_length_penalty"] != 0.0:
        raise ValueError(f"{name}: zero_over_max zeroes over-cap rewards, so profiled_length_penalty="
                         f"{p['profiled_length_penalty']} would do nothing; use constant_over_n_std or leave it 0")
    if p["profiled_length_allow_non_binary_rewards"] and not zero_over_max:
        raise ValueError(f"{name}: profiled_length_allow_non_binary_rewards only applies to zero_over_max; "
                         "every other length penalty needs binary rewards")
    if p["length_type"] == "all_generated_tokens":
        split = [k for k in ("reasoning_bonus", "answer_bonus", "longest_reasoning_penalty",
                             "longest_answer_penalty", "group_reasoning_length_penalty_coeff",
                             "group_answer_length_penalty_coeff") if p[k] > 0]
        for ch in ("reasoning", "answer"):
            if p[f"{ch}_zmad_threshold"] > 0 and p[f"{ch}_zmad_penalty"] != 0:
                split.append(f"{ch}_zmad_threshold")
            if p[f"profile_band_{ch}"]:
                split.append(f"profile_band_{ch}")
        if p["group_length_penalty_profile_gate"] and p["group_length_penalty_profile_gate_channel"] != "total":
            split.append("group_length_penalty_profile_gate_channel")
        if split:
            raise ValueError(f"{name}: length_type all_generated_tokens has no reasoning / answer split, so it "
                             f"cannot drive {split}; use total-length settings or length_type tokens / chars")


class LengthPenaltyConfig:
    """Validated ``grpo.length_penalty`` block: ``verbose``, ``default``,
    ``agent_overrides`` (agent -> partial settings, or ``None`` for the
    defaults) and ``profile_band`` (``{enabled, defaults: {channel: {a, b,
    f}}}``; channels listed there are switched on unless ``default`` sets
    the matching ``profile_band_<channel>`` itself)."""

    def __init__(self, cfg: Optional[dict] = None):
        cfg = dict(cfg or {})
        unknown = set(cfg) - {"verbose", "default", "agent_overrides", "profile_band"}
        if unknown:
            raise ValueError(f"grpo.length_penalty: unknown keys {sorted(unknown)}")
        self.verbose = bool(cfg.get("verbose", False))
        default = dict(cfg.get("default") or {})
        LengthPenaltyParams.check_keys(default, "default")
        self.overrides: Optional[dict[str, Optional[dict]]] = None
        if cfg.get("agent_overrides") is not None:
            self.overrides = {}
            for agent, ov in cfg["agent_overrides"].items():
                if ov is not None:
                    LengthPenaltyParams.check_keys(ov, f"agent_overrides.{agent}")
                self.overrides[str(agent)] = None if ov is None else dict(ov)
        self.global_band: dict[str, dict] = {}
        pb = cfg.get("profile_band")
        if pb is not None:
            if set(pb) - {"enabled", "defaults"}:
                raise ValueError(f"grpo.length_penalty.profile_band: unknown keys {sorted(set(pb) - {'enabled', 'defaults'})}")
            defaults = pb.get("defaults") or {}
            if set(defaults) - set(CHANNELS):
                raise ValueError(f"profile_band.defaults: unknown channels {sorted(set(defaults) - set(CHANNELS))}")
            bands = {ch: _check_band_channel(v, f"profile_band.defaults.{ch}") for ch, v in defaults.items()
                     if v is not None}
            if pb.get("enabled", False):
                self.global_band = bands
        self.default = dataclasses.asdict(LengthPenaltyParams(**default))
        for ch in self.global_band:
            if f"profile_band_{ch}" not in default:
                self.default[f"profile_band_{ch}"] = True
        self.default_enabled_explicit = default.get("enabled", True)
        for name, p in [("default", self.default)] + [
                (f"agent {a!r} (default merged with its override)", self.params_for(a)) for a in self.overrides or {}]:
            if p["enabled"]:
                _check_resolved(name, p)

    @property
    def active(self) -> bool:
        return bool(self.default["enabled"] or self.overrides or self.global_band)

    def params_for(self, agent: str) -> dict:
        p = dict(self.default)
        if self.overrides is not None and self.overrides.get(agent) is not None:
            p.update(self.overrides[agent])
        return p

    def band_for(self, row_band: Optional[dict]) -> Optional[dict]:
        """The row's per-prompt band over the global defaults (row channels win)."""
        if not self.global_band:
            return row_band
        merged = dict(self.global_band)
        merged.update(row_band or {})
        return merged


# ---------------------------------------------------------------- lengths
def split_reasoning_answer(row: dict) -> tuple[str, str]:
    """(reasoning text, answer text) of one rollout.

    A Responses-API ``response.output`` list (``reasoning`` items' summary
    text; ``message`` items of role assistant or none) wins when present.
    Otherwise the assistant messages of ``message_log`` are read: text inside
    ``<think>...</think>`` is reasoning, the rest answer.  Environment
    observations (user / tool / environment roles) never count."""
    resp = row.get("response")
    if isinstance(resp, dict) and isinstance(resp.get("output"), list):
        reasoning, answer = [], []
        for item in resp["output"]:
            kind = item.get("type", "")
            if kind == "reasoning":
                reasoning += [s.get("text", "") for s in item.get("summary", [])]
            elif kind == "message" and item.get("role") in (None, "assistant"):
                content = item.get("content", [])
                if isinstance(content, str):
                    answer.append(content)
                else:
                    answer += [c.get("text", "") for c in content]
        return "".join(reasoning), "".join(answer)
    reasoning, answer = [], []
    for m in row.get("message_log") or []:
        if m.get("role") != "assistant":
            continue
        text = m.get("content") or ""
        reasoning += _THINK.findall(text)
        answer.append(_THINK.sub("", text).replace("</think>", ""))
    return "".join(reasoning), "".join(answer)


def _generated_tokens(row: dict) -> int:
    if "generated_tokens" in row:
        return int(row["generated_tokens"])
    return sum(len(m["token_ids"]) for m in row.get("message_log") or [] if m.get("role") == "assistant")


def _measure(row: dict, length_type: str, tokenizer) -> dict[str, int]:
    if length_type == "all_generated_tokens":
        return {"reasoning": 0, "answer": 0, "total": _generated_tokens(row)}
    r, a = split_reasoning_answer(row)
    if length_type == "tokens" and tokenizer is not None:
        rl = len(tokenizer.encode(r, add_special_tokens=False)) if r else 0
        al = len(tokenizer.encode(a, add_special_tokens=False)) if a else 0
    else:
        rl, al = len(r), len(a)
    return {"reasoning": rl, "answer": al, "total": rl + al}


# ----------------------------------------------------------- group maths
def _relative_weights(lengths: list[int]) -> list[float]:
    lo, hi = min(lengths), max(lengths)
    if lo == hi:
        return [0.0] * len(lengths)
    raw = [1.0 - (L - lo) / (hi - lo) for L in lengths]
    mean = sum(raw) / len(raw)
    return [w - mean for w in raw]


def _zmad_outliers(lengths: list[int], z: float) -> list[int]:
    if len(lengths) < 2:
        return []
    med = statistics.median(lengths)
    mad = statistics.median([abs(x - med) for x in lengths])
    if mad == 0 or mad / max(med, 1e-9) < _ZMAD_MIN_MAD_REL:
        return []
    return [k for k, x in enumerate(lengths) if 0.6745 * (x - med) / mad > z]


def _first_extreme(cands: list[tuple[int, int]], longest: bool) -> int:
    """Index of the shortest / longest candidate (first one on ties)."""
    best = cands[0]
    for c in cands[1:]:
        if (c[1] > best[1]) if longest else (c[1] < best[1]):
            best = c
    return best[0]


def _group_adjustments(rewards: list[float], lens: list[dict[str, int]], p: dict) -> tuple[list[float], dict]:
    """Bonuses, longest penalties, group-relative scaling and zMAD of one
    group: one summed adjustment per rollout, plus the per-channel parts."""
    n = len(rewards)
    adj = [0.0] * n
    parts = {k: [0.0] * n for k in ("bonus", "longest", "relative", "zmad")}
    pos = [i for i in range(n) if rewards[i] > 0]
    if n < 2 or len(pos) < 2:
        return adj, parts
    running = list(rewards)
    ranked = sorted((rewards[i] for i in pos), reverse=True)
    top_thr = ranked[max(0, int(len(pos) * p["top_percentile"]) - 1)]
    top = [i for i in pos if rewards[i] >= top_thr]

    def add(i: int, v: float, part: str) -> None:
        running[i] += v
        adj[i] += v
        parts[part][i] += v

    for ch in CHANNELS:
        bonus = p[f"{ch}_bonus"]
        if bonus > 0:
            cands = [(i, lens[i][ch]) for i in pos if lens[i][ch] > 0]
            if cands:
                i = _first_extreme(cands, longest=False)
                if running[i] >= top_thr:
                    add(i, bonus, "bonus")
    for ch in CHANNELS:
        pen = p[f"longest_{ch}_penalty"]
        if pen > 0:
            cands = [(i, lens[i][ch]) for i in top if lens[i][ch] > 0]
            if len(cands) >= 2:
                add(_first_extreme(cands, longest=True), -pen, "longest")
    coeffs = {ch: p[f"group_{ch}_length_penalty_coeff"] for ch in CHANNELS}
    if any(c > 0 for c in coeffs.values()):
        w = {ch: _relative_weights([lens[i][ch] for i in pos]) for ch in CHANNELS}
        for k, i in enumerate(pos):
            v = sum(w[ch][k] * coeffs[ch] for ch in CHANNELS)
            if v != 0:
                add(i, v, "relative")
    for ch in CHANNELS:
        z, pen = float(p[f"{ch}_zmad_threshold"]), float(p[f"{ch}_zmad_penalty"])
        if z > 0 and pen != 0:
            for k in _zmad_outliers([lens[i][ch] for i in pos], z):
                add(pos[k], -pen, "zmad")
    return adj, parts


def _gate_open(band: Optional[dict], p: dict, rewards: list[float], lens: list[dict[str, int]]) -> tuple[bool, str]:
    """Profile gate of the group-relative coefficients (fails closed)."""
    if not p["group_length_penalty_profile_gate"]:
        return True, "disabled"
    ch, field = p["group_length_penalty_profile_gate_channel"], p["group_length_penalty_profile_gate_field"]
    block = band.get(ch) if isinstance(band, dict) else None
    limit = block.get(field) if isinstance(block, dict) else None
    if isinstance(limit, bool) or not isinstance(limit, (int, float)):
        return False, "missing_profile_limit"
    vals = [L[ch] for r, L in zip(rewards, lens) if r > 0 or not p["group_length_penalty_profile_gate_positive_only"]]
    if not vals:
        return False, "no_lengths"
    return (True, "mean_gt_limit") if statistics.mean(vals) > float(limit) else (False, "mean_le_limit")


def _profiled(row: dict, p: dict, agent: str, totals: list[int]) -> list[float]:
    """-penalty past mean + n_std * std (constant_over_n_std) or -inf past the
    longest passing profiled length (zero_over_max); 0 otherwise."""
    out = [0.0] * len(totals)
    kind = p["profiled_length_penalty_type"]
    if kind == "constant_over_n_std" and p["profiled_length_penalty"] <= 0.0:
        return out
    pr, pl = row.get("profiled_rewards"), row.get("profiled_output_lengths")
    if not isinstance(pr, list) or not isinstance(pl, list) or len(pr) != len(pl):
        raise ValueError(f"profiled_length_penalty_type {kind} is on for agent {agent!r}: every row needs top-level "
                         f"profiled_rewards and profiled_output_lengths lists of equal length, got {pr!r} and {pl!r}")
    passing = [L for r, L in zip(pr, pl) if r > p["profiled_reward_correct_threshold"]]
    if not passing or len(passing) < p["profiled_length_min_samples"]:
        return out
    if kind == "constant_over_n_std":
        thr = statistics.mean(passing) + p["profiled_length_n_std"] * (
            statistics.stdev(passing) if len(passing) >= 2 else 0.0)
        return [-p["profiled_length_penalty"] if L >= thr else 0.0 for L in totals]
    cap = max(passing)
    return [-math.inf if L > cap else 0.0 for L in totals]


def _band_multiplier(length: int, ch: Optional[dict]) -> float:
    if not ch or ch.get("a") is None or ch.get("b") is None or ch.get("f") is None or ch["b"] <= ch["a"]:
        return 1.0
    a, b, f = float(ch["a"]), float(ch["b"]), float(ch["f"])
    if length <= a:
        return 1.0
    if length >= b:
        return f
    return 1.0 - (length - a) / (b - a) * (1.0 - f)


def _is_binary(v: float) -> bool:
    return abs(v) <= _BINARY_TOL or abs(v - 1.0) <= _BINARY_TOL


_WARNED: set[str] = set()


def apply_group_length_penalties(rows: list[dict], cfg, group_size: int, tokenizer=None) -> dict[str, float]:
    """Adjust ``row["reward"]`` in place for every row; rows come in
    ``group_size`` contiguous rows per prompt.  A row carries ``reward``,
    ``agent`` (the key of ``agent_overrides``), ``message_log`` or
    ``response``, and optionally ``reward_components``, ``profiled_rewards``,
    ``profiled_output_lengths``, ``profile_band``, ``low_effort_applied``.
    Returns the ``length_penalty/*`` metrics (per-row means), or ``{}`` when
    the block enables nothing."""
    cfg = cfg if isinstance(cfg, LengthPenaltyConfig) else LengthPenaltyConfig(cfg)
    if not cfg.active or not rows:
        return {}
    if group_size <= 0:
        raise ValueError("group_size must be greater than zero")
    n = len(rows)
    orig = [float(r["reward"]) for r in rows]
    group_adj = [0.0] * n
    prof_adj = [0.0] * n
    rate_adj = [0.0] * n
    lens = [{"reasoning": 0, "answer": 0, "total": 0} for _ in range(n)]
    binary_ok = [False] * n
    skipped_non_binary = 0
    band_groups: list[tuple[int, int, dict, Optional[dict]]] = []
    notes: dict[int, str] = {}
    for g in range(0, n, group_size):
        m = min(group_size, n - g)
        rg = range(g, g + m)
        agent = str(rows[g].get("agent", ""))
        p = cfg.params_for(agent)
        if not p["enabled"]:
            notes[g] = "disabled"
            continue
        has_components = any(rows[i].get("reward_components") for i in rg)
        zero_over_max = p["profiled_length_penalty_type"] == "zero_over_max"
        if zero_over_max and has_components:
            raise ValueError(f"zero_over_max is on for agent {agent!r}, which produced multi-component rewards: "
                             "zeroing the scalar would break reward == sum(reward_components); turn it off for "
                             "this agent under agent_overrides")
        binary = not has_components and all(_is_binary(orig[i]) for i in rg)
        cap_only = not binary and zero_over_max and p["profiled_length_allow_non_binary_rewards"]
        if not binary and not cap_only:
            skipped_non_binary += m
            if agent not in _WARNED:
                _WARNED.add(agent)
                log.warning("length penalties need binary (0/1) single-reward rewards; agent %r produced others, "
                            "its groups are left unadjusted", agent)
            notes[g] = "non_binary"
            continue
        if binary:
            for i in rg:
                binary_ok[i] = True
        if any(rows[i].get("low_effort_applied") for i in rg):
            notes[g] = "low_effort"
            continue
        if cap_only and any(orig[i] < 0 for i in rg):
            raise ValueError(f"agent {agent!r} produced a negative reward ({min(orig[i] for i in rg)}); "
                             "profiled_length_allow_non_binary_rewards cannot zero over-cap rollouts above it")
        for i in rg:
            lens[i] = _measure(rows[i], p["length_type"], tokenizer)
        totals = [lens[i]["total"] for i in rg]
        if cap_only:
            prof_adj[g:g + m] = _profiled(rows[g], p, agent, totals)
            notes[g] = "cap_only"
            continue
        band = cfg.band_for(rows[g].get("profile_band"))
        rewards = orig[g:g + m]
        is_open, why = _gate_open(band, p, rewards, lens[g:g + m])
        q = dict(p)
        if not is_open:
            for ch in CHANNELS:
                q[f"group_{ch}_length_penalty_coeff"] = 0.0
        adj, _ = _group_adjustments(rewards, lens[g:g + m], q)
        group_adj[g:g + m] = adj
        prof_adj[g:g + m] = _profiled(rows[g], p, agent, totals)
        w = p["pass_rate_length_penalty_weight"]
        correct = [i for i in rg if orig[i] > 0]
        if w > 0.0 and correct:
            rho = len(correct) / m
            l_max = float(max(lens[i]["total"] for i in correct))
            if l_max > 0.0:
                for i in correct:
                    rate_adj[i] = -w * rho * lens[i]["total"] / l_max
        band_groups.append((g, m, p, band))
        notes[g] = f"gate={why}"
    base = [0.0] * n
    for i, row in enumerate(rows):
        if not binary_ok[i] and prof_adj[i] != -math.inf:
            continue
        # the constant profiled penalty does not stack on a rollout that the
        # group-relative channels already pushed down; the zero_over_max cap always applies
        pa = 0.0 if (group_adj[i] < 0 and prof_adj[i] != -math.inf) else prof_adj[i]
        base[i] = max(0.0, orig[i] + group_adj[i] + pa + rate_adj[i])
        row["reward"] = base[i]
    for g, m, p, band in band_groups:
        if not band:
            continue
        chans = [(ch, band.get(ch)) for ch in ("total", "reasoning", "answer") if p[f"profile_band_{ch}"]]
        if not chans:
            continue
        for i in range(g, g + m):
            if not binary_ok[i] or orig[i] <= 0 or base[i] <= 0:
                continue
            r = base[i]
            for ch, block in chans:
                r *= _band_multiplier(lens[i][ch], block)
            rows[i]["reward"] = r
    final = [float(r["reward"]) for r in rows]
    if cfg.verbose:
        for g in range(0, n, group_size):
            m = min(group_size, n - g)
            print(f"[length_penalty] group {g // group_size} agent={rows[g].get('agent', '')!r} "
                  f"{notes.get(g, '')} rewards {orig[g:g + m]} -> {[round(x, 4) for x in final[g:g + m]]} "
                  f"total_len {[lens[i]['total'] for i in range(g, g + m)]}", flush=True)
    return {
        "length_penalty/env_reward_mean": sum(orig) / n,
        "length_penalty/reward_delta_mean": sum(f - o for f, o in zip(final, orig)) / n,
        "length_penalty/wiped_correct_frac": sum(1 for f, o in zip(final, orig) if o > 0 and f <= 0.0) / n,
        "length_penalty/adjusted_frac": sum(1 for f, o in zip(final, orig) if f != o) / n,
        "length_penalty/skipped_non_binary_frac": skipped_non_binary / n,
    }


def _agent_key(info: Any, task: Optional[str]) -> str:
    if isinstance(info, dict):
        ref = info.get("agent_ref")
        if isinstance(ref, dict) and ref.get("name"):
            return str(ref["name"])
        tid = info.get("task_id")
        if isinstance(tid, dict) and tid.get("taskset"):
            return str(tid["taskset"])
    return str(task or "")


_ROW_FIELDS = ("profiled_rewards", "profiled_output_lengths", "profile_band", "reward_components",
               "low_effort_applied", "response")


def apply_length_penalty_to_rollout(rollout, cfg, group_size: int, tokenizer=None) -> dict[str, float]:
    """Apply ``grpo.length_penalty`` to a rollout batch (``message_log``,
    ``total_reward``, ``extra_env_info``, ``task_name``): the reward before
    the adjustment is kept as ``env_reward`` and ``total_reward`` is
    replaced.  Per-prompt fields are read from the top level of each row's
    ``extra_env_info``; the agent key is its ``agent_ref.name``, else its
    ``task_id.taskset``, else the row's task name."""
    cfg = cfg if isinstance(cfg, LengthPenaltyConfig) else LengthPenaltyConfig(cfg)
    if not cfg.active:
        return {}
    tr = rollout["total_reward"]
    B = len(rollout["message_log"])
    infos = rollout["extra_env_info"] if "extra_env_info" in rollout else [None] * B
    tasks = rollout["task_name"] if "task_name" in rollout else [None] * B
    rows = []
    for b in range(B):
        info = infos[b] if isinstance(infos[b], dict) else {}
        row = {"reward": float(tr[b]), "agent": _agent_key(info, tasks[b]), "message_log": rollout["message_log"][b]}
        for k in _ROW_FIELDS:
            if k in info:
                row[k] = info[k]
        rows.append(row)
    metrics = apply_group_length_penalties(rows, cfg, group_size, tokenizer)
    rollout["env_reward"] = tr.clone()
    rollout["total_reward"] = torch.tensor([r["reward"] for r in rows], dtype=tr.dtype)
    return metrics
