"""The in-tree native extension, when built, must import (catches unresolved symbols on CPU)."""

import glob
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_extension_imports_when_built():
    if not glob.glob(os.path.join(ROOT, "rl_b200", "_C*.so")):
        pytest.skip("extension not built")
    from rl_b200.ops import _ext

    assert _ext.has_ext(), repr(_ext._ERR)
    for name in ("gemm_nt", "flash_attn_fwd", "flash_attn_bwd", "paged_decode_attn", "sample", "adamw_step",
                 "logprob_partials", "rmsnorm_fwd", "quant_fp8_block", "moe_router_topk", "nvls_all_reduce",
                 "nvls_reduce_shard", "dp_wait_ready", "bounds_errors", "debug_bounds_build"):
        assert hasattr(_ext.ext()._mod, name)
