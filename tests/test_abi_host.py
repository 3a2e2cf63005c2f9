"""Host-side checks that need no GPU: the C-ABI library loads and exports
every entry point include/dial_b200.h declares; topology parsing; the
product's synthetic generator agrees with the oracle's; argument validation
that fails before any device work."""

import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "dial_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dial_b200_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_surface():
    names = declared_functions()
    for must in ["dial_b200_abi_version", "dial_b200_qlinear_forward", "dial_b200_w8a16_from_dense",
                 "dial_b200_qlinear_create", "dial_b200_layer_forward", "dial_b200_range_forward",
                 "dial_b200_decode_step", "dial_b200_session_reset"]:
        assert must in names


def test_library_exports_every_declared_symbol():
    from dial_b200 import _abi

    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s+(dial_b200_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding covers the whole surface too
    assert set(declared_functions()) <= set(_abi.exported_symbols())


def test_abi_version_without_gpu():
    from dial_b200 import _abi

    assert _abi.lib.dial_b200_abi_version() == _abi.ABI_VERSION == 2


def test_null_handles_are_rejected_without_device_work():
    from dial_b200 import _abi

    assert _abi.lib.dial_b200_qlinear_in_dim(None) == -1
    assert _abi.lib.dial_b200_step_kernel_count(None, 1) == -1
    buf = C.create_string_buffer(256)
    rc = _abi.lib.dial_b200_qlinear_forward(None, None, None, 1, None, buf, 256)
    assert rc == _abi.DIAL_ERR_INVALID and b"null" in buf.value
    rc = _abi.lib.dial_b200_decode_loop_run(None, 1, 1, buf, 256)
    assert rc == _abi.DIAL_ERR_INVALID


def test_synth_table_matches_oracle():
    import dial_oracle as O
    from dial_b200.synth import normal_table_bits

    mine = normal_table_bits(0.02)
    ref = O.bf16_bits(O.normal_table(0.02))
    assert np.array_equal(mine, ref)
    assert abs(float(O.normal_table(0.02).std()) - 0.02) < 5e-4


def test_topology_range_expansion_and_stages():
    from dial_b200.topology import Topology, TopologyError

    t = Topology.from_yaml("""
worker0:
  host: '192.168.1.87:10120'
  description: 'first'
  layers:
    - 'model.layers.0-17'
worker1:
  host: '10.0.0.2:10120'
  layers: ['model.layers.18-35']
""")
    assert len(t.nodes["worker0"].layers) == 18
    assert t.get_node_for_layer("model.layers.20")[0] == "worker1"
    assert t.get_node_for_layer("model.layers.40") is None
    assert t.nodes["worker0"].is_layer_owner("model.layers.3.self_attn")
    assert t.stages(36) == [("worker0", 0, 18), ("worker1", 18, 18)]
    with pytest.raises(TopologyError, match="end must be > start"):
        Topology.from_yaml("w:\n  host: h\n  layers: ['model.layers.5-5']\n")
    with pytest.raises(TopologyError):
        Topology.from_yaml("w:\n  host: h\n  layers: ['model.layers.0-3']\n").stages(8)
    even = Topology.even_split(36, 8)
    assert [c for _, _, c in even.stages(36)] == [5, 5, 5, 5, 4, 4, 4, 4]
    assert Topology.from_yaml("{}").stages(36) == []


def test_reference_topology_file_parses():
    from dial_b200.topology import Topology

    t = Topology.from_yaml("worker0:\n  host: '192.168.1.87:10120'\n  description: '87 server'\n"
                           "  layers:\n    - 'model.layers.0-31'\n")
    assert t.stages(32) == [("worker0", 0, 32)]
