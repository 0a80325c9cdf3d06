"""The C ABI library loads on a machine without a GPU and exports every
function include/zs.h declares; pure-host helpers answer without a device."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "zs.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zs_\w+)\s*\(", text)))


def test_library_builds_and_exports_all_header_symbols():
    from zs_b200 import build, _lib

    build.build()
    lib = _lib.lib()
    names = header_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(_lib.exported_symbols()) == names


def test_host_only_entry_points():
    from zs_b200 import _lib

    lib = _lib.lib()
    assert lib.zs_version() >= 1
    assert lib.zs_error_string(0) == b"ok"
    assert b"workspace" in lib.zs_error_string(6)
    assert lib.zs_flatten_sort_count_workspace(131072, 64) == 32 * 65 * 4
    assert lib.zs_scatter2scatter_workspace(100, 64, 1, 1) == 0
    assert lib.zs_scatter2scatter_workspace(100, 64, 1, 0) >= 100 * 128
    # copy-engine all-reduce chunking: ceil(count / world) rounded up to 8 elements
    assert lib.zs_ipc_handle_size() == 64
    assert lib.zs_ce_allreduce_chunk(9, 2) == 8 and lib.zs_ce_allreduce_chunk(1_000_003, 2) == 500_008
    assert lib.zs_ce_allreduce_chunk(16, 4) == 8 and lib.zs_ce_allreduce_chunk(0, 2) == 0
    assert lib.zs_muonmd_pre_workspace(64, 1536, 1536) >= 4 * (64 * 1536 * 6 + 64 * 24 * 1536 + 64 * 24 * 6)


def test_ops_refuse_cpu_tensors():
    import torch

    from scattermoe.kernels import ops
    from zs_b200 import ZsError

    x = torch.zeros(4, 8)
    with pytest.raises(ZsError):
        ops.rowwise_sum_product(torch.zeros(2, 2, 8), torch.zeros(2, 8))
    with pytest.raises(ZsError):
        ops.group(x, torch.zeros(4, dtype=torch.long))
