"""Environment registry and the non-math environments.

Reference environments (``nemo_rl/environments/``): math verification
(``math_environment.py:448``), code execution, games (sliding puzzle), a reward-
model environment and the NeMo-Gym bridge.  Here:

* ``CodeEnvironment`` - runs the extracted Python code block of the response in
  a separate interpreter process (resource/time-limited) against the sample's
  test snippet; reward 1.0 when it exits cleanly.
* ``SlidingPuzzleEnvironment`` - multi-turn game: the model answers with moves
  (``up``/``down``/``left``/``right``); observations carry the board; reward 1.0
  when solved, episodes end on solve or move budget.
* ``RewardModelEnvironment`` - scores (prompt, response) with a reward-model
  policy worker (``num_labels: 1``): reward = value at the last token.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
import tempfile
from typing import Any, Callable, Optional

import torch

from rl_b200.environments.interfaces import EnvironmentInterface, EnvironmentReturn

__all__ = ["CodeEnvironment", "SlidingPuzzleEnvironment", "RewardModelEnvironment", "make_environment",
           "register_environment"]

_REGISTRY: dict[str, Callable[..., EnvironmentInterface]] = {}


def register_environment(name: str, factory: Callable[..., EnvironmentInterface]) -> None:
    _REGISTRY[name] = factory


def make_environment(name: str, cfg: Optional[dict] = None, **kw) -> EnvironmentInterface:
    if name not in _REGISTRY:
        raise KeyError(f"unknown environment {name!r}; registered: {sorted(_REGISTRY)}")
    return _REGISTRY[name](cfg or {}, **kw)


def _text(log: list[dict], decode) -> str:
    parts = []
    for m in log:
        if m["role"] != "assistant":
            continue
        parts.append(m.get("content") or (decode(m["token_ids"].tolist()) if decode else ""))
    return "".join(parts)


class CodeEnvironment(EnvironmentInterface):
    _BLOCK = re.compile(r"```(?:python)?\n(.*?)```", re.S)

    def __init__(self, cfg: Optional[dict] = None, decode=None):
        self.cfg = cfg or {}
        self.decode = decode
        self.timeout = float(self.cfg.get("timeout_s", 5.0))

    def run_code(self, code: str, tests: str) -> bool:
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "prog.py")
            with open(path, "w") as f:
                f.write(code + "\n\n" + (tests or ""))
            try:
                r = subprocess.run([sys.executable, "-I", path], cwd=d, capture_output=True, timeout=self.timeout,
                                   env={"PATH": os.environ.get("PATH", "")})
                return r.returncode == 0
            except subprocess.TimeoutExpired:
                return False

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        rewards = []
        for log, meta in zip(message_log_batch, metadata):
            txt = _text(log, self.decode)
            m = self._BLOCK.findall(txt)
            code = m[-1] if m else txt
            rewards.append(1.0 if self.run_code(code, (meta or {}).get("tests", "")) else 0.0)
        n = len(rewards)
        return EnvironmentReturn([{"role": "environment", "content": ""}] * n, list(metadata), [None] * n,
                                 torch.tensor(rewards), torch.ones(n, dtype=torch.bool), [None] * n)


class SlidingPuzzleEnvironment(EnvironmentInterface):
    """N x N sliding puzzle; metadata holds ``board`` (list of lists, 0 = blank)."""

    MOVES = {"up": (-1, 0), "down": (1, 0), "left": (0, -1), "right": (0, 1)}

    def __init__(self, cfg: Optional[dict] = None, decode=None):
        self.cfg = cfg or {}
        self.decode = decode
        self.max_moves = int(self.cfg.get("max_moves", 50))

    @staticmethod
    def solved(board) -> bool:
        flat = [x for row in board for x in row]
        return flat == list(range(1, len(flat))) + [0]

    def apply(self, board, move: str):
        n = len(board)
        r, c = next((i, j) for i in range(n) for j in range(n) if board[i][j] == 0)
        dr, dc = self.MOVES[move]
        rr, cc = r + dr, c + dc
        if not (0 <= rr < n and 0 <= cc < n):
            return board, False
        b = [row[:] for row in board]
        b[r][c], b[rr][cc] = b[rr][cc], b[r][c]
        return b, True

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        obs, meta_out, rewards, done = [], [], [], []
        for log, meta in zip(message_log_batch, metadata):
            meta = dict(meta or {})
            board = meta.get("board")
            last = [m for m in log if m["role"] == "assistant"][-1:]
            text = (last[0].get("content") or (self.decode(last[0]["token_ids"].tolist()) if self.decode else "")) \
                if last else ""
            moves = re.findall(r"\b(up|down|left|right)\b", text.lower())
            used = int(meta.get("moves_used", 0))
            for mv in moves:
                if used >= self.max_moves:
                    break
                board, _ = self.apply(board, mv)
                used += 1
            meta.update(board=board, moves_used=used)
            ok = self.solved(board)
            rewards.append(1.0 if ok else 0.0)
            done.append(ok or used >= self.max_moves)
            obs.append({"role": "environment", "content": "solved" if ok else
                        "board:\n" + "\n".join(" ".join(str(x) for x in row) for row in board)})
            meta_out.append(meta)
        n = len(rewards)
        return EnvironmentReturn(obs, meta_out, [None] * n, torch.tensor(rewards), torch.tensor(done), [None] * n)


class RewardModelEnvironment(EnvironmentInterface):
    def __init__(self, cfg: Optional[dict] = None, reward_model=None):
        self.cfg = cfg or {}
        self.rm = reward_model

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        from rl_b200.data.llm_message_utils import batched_message_log_to_flat_message
        from rl_b200.distributed.batched_data_dict import BatchedDataDict

        flat, lengths = batched_message_log_to_flat_message(message_log_batch)
        vals = self.rm.get_values(BatchedDataDict({"input_ids": flat["token_ids"], "input_lengths": lengths}))["values"]
        r = vals.gather(1, (lengths - 1).clamp_min(0).unsqueeze(1)).squeeze(1)
        n = len(message_log_batch)
        return EnvironmentReturn([{"role": "environment", "content": ""}] * n, list(metadata), [None] * n, r.float(),
                                 torch.ones(n, dtype=torch.bool), [None] * n)


def _register_defaults():
    from rl_b200.environments.math_environment import MathEnvironment
    from rl_b200.environments.synthetic import EvenTokenEnvironment, HashRewardEnvironment

    register_environment("math", lambda c, **k: MathEnvironment(c, **k))
    register_environment("hash", lambda c, **k: HashRewardEnvironment(c))
    register_environment("even", lambda c, **k: EvenTokenEnvironment(c))
    register_environment("code", lambda c, **k: CodeEnvironment(c, **k))
    from rl_b200.environments.http_gym import HttpGymEnvironment

    register_environment("http_gym", lambda c, **k: HttpGymEnvironment(c))
    register_environment("nemo_gym", lambda c, **k: HttpGymEnvironment(c))
    register_environment("sliding_puzzle", lambda c, **k: SlidingPuzzleEnvironment(c, **k))
    register_environment("reward_model", lambda c, **k: RewardModelEnvironment(c, **k))
    from rl_b200.environments import verifiers

    verifiers.register(register_environment)


_register_defaults()
