"""C-ABI checks that need no GPU: libkvm.so loads, exports every function that
include/kvm.h declares (and the binding knows all of them), and the ctypes
structs have the C layout."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kvm.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(kvm_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "kvm_session_create" in names and "kvm_step" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    import kvm
    kvm.build()
    lib = C.CDLL(kvm.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", kvm.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (kvm_\w+)$", out, flags=re.M))
    assert exported == set(declared_functions())
    assert set(kvm.ABI_SYMBOLS) == set(declared_functions())


def test_host_only_calls_without_gpu():
    import kvm
    L = kvm.lib()
    c = kvm.Config()
    L.kvm_config_default(C.byref(c))
    assert c.block_tokens == 128 and c.sink_blocks == 1 and c.type_k == kvm.TYPE_Q8_0
    assert kvm.row_bytes(kvm.TYPE_Q8_0, 1024) == 1088
    assert kvm.row_bytes(kvm.TYPE_Q4_0, 1024) == 576
    assert kvm.row_bytes(kvm.TYPE_Q5_0, 1024) == 704
    assert kvm.row_bytes(kvm.TYPE_F16, 1024) == 2048
    # invalid configurations are rejected before any device work
    h = C.c_void_p()
    bad = kvm.default_config(max_blocks=0)
    assert L.kvm_session_create(C.byref(bad), 0, C.byref(h)) == kvm.KVM_EINVAL
    assert b"max_blocks" in L.kvm_last_error(None)
    bad = kvm.default_config(type_k=3)
    assert L.kvm_session_create(C.byref(bad), 0, C.byref(h)) == kvm.KVM_EINVAL
    bad = kvm.default_config(n_head_kv=3, head_dim=10)
    assert L.kvm_session_create(C.byref(bad), 0, C.byref(h)) == kvm.KVM_EINVAL
    assert L.kvm_session_create(None, 0, C.byref(h)) == kvm.KVM_EINVAL


def test_row_quantizers_reject_odd_destinations_before_any_launch():
    """An odd d_dst would reach 2-byte device stores; both row quantizers
    return KVM_EINVAL first (the pointers are never dereferenced or launched
    on, so this runs without a GPU)."""
    import kvm
    L = kvm.lib()
    src, odd = 0x10000, 0x20001
    for fn in (L.kvm_quantize_rows, L.kvm_quantize_rows_noalloc):
        assert fn(None, kvm.TYPE_Q8_0, src, 4, 1024, odd) == kvm.KVM_EINVAL
        assert b"2-byte aligned" in L.kvm_last_error(None)
        assert fn(None, kvm.TYPE_Q8_0, src + 8, 4, 1024, 0x20000) == kvm.KVM_EINVAL


C_LAYOUT = r"""
#include <stddef.h>
#include <stdio.h>
#include "kvm.h"
#define P(T, F) printf(#T "." #F " %zu\n", offsetof(T, F))
int main(void) {
    printf("kvm_config %zu\nkvm_source %zu\nkvm_window %zu\nkvm_plan %zu\nkvm_timings %zu\n",
           sizeof(kvm_config), sizeof(kvm_source), sizeof(kvm_window), sizeof(kvm_plan),
           sizeof(kvm_timings));
    P(kvm_config, max_blocks); P(kvm_config, immutable_refresh_abs_delta_tokens);
    P(kvm_config, staging_bytes); P(kvm_source, location); P(kvm_plan, n_moves);
    P(kvm_plan, cold_to); P(kvm_plan, total_window_tokens);
    return 0;
}
"""


def test_struct_layouts_match_c():
    import kvm
    cc = os.environ.get("CC", "gcc")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(src, "w").write(C_LAYOUT)
        r = subprocess.run([cc, "-I", os.path.join(ROOT, "include"), src, "-o", exe],
                           capture_output=True, text=True)
        if r.returncode != 0:
            pytest.skip("no C compiler: " + r.stderr[:200])
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    got = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    got = {k: int(v) for k, v in got.items()}
    assert got["kvm_config"] == C.sizeof(kvm.Config)
    assert got["kvm_source"] == C.sizeof(kvm.Source)
    assert got["kvm_window"] == C.sizeof(kvm.Window)
    assert got["kvm_plan"] == C.sizeof(kvm._Plan)
    assert got["kvm_timings"] == C.sizeof(kvm.Timings)
    assert got["kvm_config.max_blocks"] == kvm.Config.max_blocks.offset
    assert got["kvm_config.immutable_refresh_abs_delta_tokens"] == \
        kvm.Config.immutable_refresh_abs_delta_tokens.offset
    assert got["kvm_config.staging_bytes"] == kvm.Config.staging_bytes.offset
    assert got["kvm_source.location"] == kvm.Source.location.offset
    assert got["kvm_plan.n_moves"] == kvm._Plan.n_moves.offset
    assert got["kvm_plan.cold_to"] == kvm._Plan.cold_to.offset
    assert got["kvm_plan.total_window_tokens"] == kvm._Plan.total_window_tokens.offset
