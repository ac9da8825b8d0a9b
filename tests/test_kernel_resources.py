"""Build check of every CUDA kernel's resources, like the reference's
kernel_resources test (cmake/check_kernel_resources.cmake:40-53): no stack
frame, no spill stores or loads (so no local memory) in any function ptxas
compiles for sm_100a. It reads the `-Xptxas -v` summaries that the library's
Makefile keeps beside each object (bonsai-ternary-fast_b200/_build/*.o.ptxas.log);
no GPU is needed."""
import glob
import os
import re

import pytest

from conftest import PKG

PROPS = re.compile(r"Function properties for (\S+)\n\s*(\d+) bytes stack frame, (\d+) bytes spill stores, "
                   r"(\d+) bytes spill loads")
ENTRY = re.compile(r"Compiling entry function '(\S+)' for 'sm_100a'")


def _logs():
    logs = sorted(glob.glob(os.path.join(PKG, "_build", "*.o.ptxas.log")))
    if not logs:
        pytest.skip("no per-object ptxas logs: build the library here with make -C bonsai-ternary-fast_b200")
    return {os.path.basename(p): open(p).read() for p in logs}


def test_every_kernel_has_no_stack_and_no_spills():
    logs = _logs()
    bad, entries, props = [], set(), {}
    for name, text in logs.items():
        entries |= set(ENTRY.findall(text))
        for fn, stack, st, ld in PROPS.findall(text):
            props[fn] = (int(stack), int(st), int(ld))
            if (int(stack), int(st), int(ld)) != (0, 0, 0):
                bad.append((name, fn, stack, st, ld))
    assert not bad, bad
    assert entries and entries <= set(props), sorted(entries - set(props))[:5]


def test_hot_path_kernels_are_in_the_build():
    text = "".join(_logs().values())
    for kernel in ("gemv_kernel", "gemm_kernel", "quant_q8_kernel", "prep_kernel", "repack_panels_kernel",
                   "gdn_mix_kernel", "attn_fused_kernel"):
        assert re.search(rf"Compiling entry function '\S*{kernel}\S*' for 'sm_100a'", text), kernel
