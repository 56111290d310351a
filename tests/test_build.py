"""Build-time checks (CPU): the ptxas resource report is parsed per kernel,
and the persistent attention kernel's register split (setmaxnreg over the
launch allocation) is refused unless it built with exactly the register
count the split assumes, without spills and without a stack frame."""

from __future__ import annotations

import pytest

import build as tk_build

LOG = """ptxas info    : Compiling entry function '_ZN2tk4attn15attn_fwd_kernelILi64EEEv14CUtensorMap_st' for 'sm_100a'
ptxas info    : Function properties for _ZN2tk4attn15attn_fwd_kernelILi64EEEv14CUtensorMap_st
    {stack} bytes stack frame, {spill} bytes spill stores, {spill} bytes spill loads
ptxas info    : Used {regs} registers, used 1 barriers, 208 bytes smem
ptxas info    : Function properties for _ZN2tk6helperEv
    48 bytes stack frame, 24 bytes spill stores, 24 bytes spill loads
ptxas info    : Compiling entry function '_ZN2tk2ln12ln_warp_rowsILi8EffffEEvNS0_4ArgsE' for 'sm_100a'
ptxas info    : Function properties for _ZN2tk2ln12ln_warp_rowsILi8EffffEEvNS0_4ArgsE
    32 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 80 registers, used 0 barriers
"""


def test_kernel_resources_parses_each_entry():
    res = tk_build.kernel_resources(LOG.format(regs=168, spill=0, stack=0))
    # a non-inlined helper's properties block after the kernel is not the kernel's
    assert res["_ZN2tk4attn15attn_fwd_kernelILi64EEEv14CUtensorMap_st"] == (168, 0, 0)
    assert res["_ZN2tk2ln12ln_warp_rowsILi8EffffEEvNS0_4ArgsE"] == (80, 0, 32)


def test_register_split_check():
    tk_build.check_register_split(LOG.format(regs=168, spill=0, stack=0))
    with pytest.raises(RuntimeError, match="register split"):
        tk_build.check_register_split(LOG.format(regs=160, spill=0, stack=0))
    with pytest.raises(RuntimeError, match="register split"):
        tk_build.check_register_split(LOG.format(regs=168, spill=12, stack=0))
    with pytest.raises(RuntimeError, match="register split"):
        tk_build.check_register_split(LOG.format(regs=168, spill=0, stack=16))
