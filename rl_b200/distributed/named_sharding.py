"""Named N-d rank layouts.

Reference: ``NamedSharding`` (``nemo_rl/distributed/named_sharding.py:31``), the
object its worker groups use to describe which ranks hold which shard
(``sharding_annotations.get_axis_size("data_parallel")`` and so on).  The
method names and their results are kept, so code written against the
reference's annotations runs unchanged; ``from_parallel_state`` builds the
layout of this framework's process grid (rank = t + tp * (c + cp * (d + dp * p))).
"""

from __future__ import annotations

from typing import Any, Sequence, Union

import numpy as np

__all__ = ["NamedSharding", "from_parallel_state", "AXES"]

# outermost to innermost, as ranks are numbered by init_distributed
AXES = ["pipeline_parallel", "data_parallel", "context_parallel", "tensor_parallel"]


class NamedSharding:
    """Ranks arranged in an N-d array whose axes have names.

    >>> s = NamedSharding([[[0, 1, 2, 3], [4, 5, 6, 7]]], ["dp", "pp", "tp"])
    >>> s.shape
    {'dp': 1, 'pp': 2, 'tp': 4}
    >>> s.get_ranks(dp=0, pp=1).layout.tolist()
    [4, 5, 6, 7]
    """

    def __init__(self, layout: Sequence[Any] | np.ndarray, names: list[str]):
        try:
            arr = np.asarray(layout)
        except ValueError as e:  # ragged nesting
            raise ValueError(f"layout is not a rectangular array: {e}") from e
        if not np.issubdtype(arr.dtype, np.integer):
            if arr.size and not np.all(np.mod(arr, 1) == 0):
                raise ValueError("layout must hold integer rank ids")
            arr = arr.astype(np.int32)
        if arr.ndim != len(names):
            raise ValueError(f"layout has {arr.ndim} dimensions but {len(names)} names were given")
        vals, counts = np.unique(arr, return_counts=True)
        if (counts > 1).any():
            raise ValueError(f"duplicate ranks in layout: {vals[counts > 1].tolist()}")
        if len(set(names)) != len(names):
            raise ValueError(f"duplicate axis names: {names}")
        self._layout = arr
        self._names = list(names)
        self._axis = {n: i for i, n in enumerate(self._names)}

    # ------------------------------------------------------------------ shape
    @property
    def shape(self) -> dict[str, int]:
        return {n: int(self._layout.shape[i]) for i, n in enumerate(self._names)}

    @property
    def names(self) -> list[str]:
        return list(self._names)

    @property
    def ndim(self) -> int:
        return self._layout.ndim

    @property
    def size(self) -> int:
        return int(self._layout.size)

    @property
    def layout(self) -> np.ndarray:
        return self._layout

    def get_axis_index(self, name: str) -> int:
        if name not in self._axis:
            raise ValueError(f"unknown axis {name!r}; axes: {self._names}")
        return self._axis[name]

    def get_axis_size(self, name: str) -> int:
        return int(self._layout.shape[self.get_axis_index(name)])

    # ----------------------------------------------------------------- lookup
    def get_worker_coords(self, worker_id: int) -> dict[str, int]:
        """Coordinate of ``worker_id`` along every axis."""
        hit = np.argwhere(self._layout == worker_id)
        if len(hit) == 0:
            raise ValueError(f"rank {worker_id} is not in this layout")
        return {n: int(hit[0][i]) for i, n in enumerate(self._names)}

    @staticmethod
    def is_axis_zero(coords: dict[str, int], axes: Sequence[str]) -> bool:
        """Whether ``coords`` is 0 along every axis of ``axes`` (missing axes count as 0)."""
        return all(coords.get(a, 0) == 0 for a in axes)

    def _index(self, coords: dict[str, int], strict: bool):
        idx: list[Any] = [slice(None)] * self.ndim
        for name, i in coords.items():
            ax = self.get_axis_index(name)
            if not 0 <= i < self._layout.shape[ax]:
                if strict:
                    raise IndexError(f"index {i} out of range for axis {name!r} of size {self._layout.shape[ax]}")
                return None
            idx[ax] = i
        return tuple(idx)

    def get_ranks_by_coord(self, **coords: int) -> list[int]:
        """Sorted ranks whose coordinates match ``coords`` (unnamed axes: any);
        [] when a coordinate is out of range."""
        idx = self._index(coords, strict=False)
        if idx is None:
            return []
        return sorted(int(x) for x in np.unique(self._layout[idx]))

    def get_ranks(self, **coords: int) -> Union["NamedSharding", int]:
        """The sub-layout at ``coords`` over the remaining axes (an int when every
        axis is fixed)."""
        idx = self._index(coords, strict=True)
        sub = self._layout[idx]
        rest = [n for n in self._names if n not in coords]
        if not rest:
            return int(sub)
        return NamedSharding(sub, rest)

    def __repr__(self) -> str:
        return f"NamedSharding(shape={self.shape}, layout={self._layout.tolist()})"

    def __eq__(self, other: object) -> bool:
        return (isinstance(other, NamedSharding) and self._names == other._names
                and np.array_equal(self._layout, other._layout))


def from_parallel_state(ps) -> NamedSharding:
    """The process grid of ``ps`` (``rl_b200.parallel.state.ParallelState``)."""
    layout = np.arange(ps.world_size, dtype=np.int32).reshape(ps.pp_size, ps.dp_size, ps.cp_size, ps.tp_size)
    return NamedSharding(layout, list(AXES))
