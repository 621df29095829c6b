"""The C-ABI library loads and exports every symbol include/glad_b200.h declares (no GPU needed)."""
import ctypes
import os
import re

from rl_quant_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "glad_b200.h")


def declared():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\**\s+\**(glad_[a-z0-9_]+)\s*\(", txt, flags=re.M))


def test_header_lists_entry_points():
    names = declared()
    assert "glad_actor_forward" in names and "glad_conv2_int8_fused" in names
    assert names == set(N.SIGNATURES), names ^ set(N.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(N.LIB_PATH)
    for name in declared():
        assert hasattr(lib, name), name
    assert N.load().glad_abi_version() == 102


def test_workspace_sizes_are_host_only():
    lib = N.load()
    assert lib.glad_qlinear_workspace_size() >= 36
    small, big = lib.glad_actor_workspace_size(1), lib.glad_actor_workspace_size(4096)
    assert 0 < small < big
    assert big >= 4096 * (187 * 16 + 224 * 2)
