"""gkv_select_tiers_static: tier selection with the library's own scratch.

Some callers cannot allocate device memory at the moment they select tiers --
an engine that has already given all free device memory to its own pool, or a
latency-critical path that cannot pay for cudaMalloc's implicit device-wide
synchronisation.  For them the library offers this entry point, which takes no
workspace and allocates nothing; it keeps the selection workspace (13 bytes per
token) in a fixed 13 MiB device array (up to GKV_STATIC_SELECT_MAX_TOKENS tokens).

These tests call it through the C ABI and check, on two calls in a row, that
its index lists equal those of gkv_select_tiers with a caller-supplied
workspace (integer outputs: exact equality).  This file sorts last so that a
run stopping at its first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from graphkv_b200 import _lib as L
from graphkv_b200.config import resolve_tiers
from graphkv_b200.profiles import get_profile

pytestmark = pytest.mark.gpu


def _select(static: bool, scores: torch.Tensor, tiers) -> torch.Tensor:
    lib = L.lib()
    dev = scores.device
    T = tiers.seq_len
    idx = torch.full((T,), -1, dtype=torch.int32, device=dev)
    r, s, c = torch.split(idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
    pol = tiers.policy()
    st = L.stream_handle(dev)
    if static:
        status = lib.gkv_select_tiers_static(scores.data_ptr(), None, ctypes.byref(pol), r.data_ptr(), s.data_ptr(),
                                             c.data_ptr(), st)
    else:
        ws = torch.empty(int(lib.gkv_select_workspace_bytes(T)), dtype=torch.uint8, device=dev)
        status = lib.gkv_select_tiers(scores.data_ptr(), None, ctypes.byref(pol), r.data_ptr(), s.data_ptr(),
                                      c.data_ptr(), ws.data_ptr(), ws.numel(), st)
    L.check(status)
    torch.cuda.synchronize(dev)
    return idx.cpu()


@pytest.mark.parametrize("T,profile,kind", [
    (32768, "graphkv", "lognormal"),
    (9000, "graphkv-qwen7-nf4", "lognormal"),
    (131072, "graphkv", "lognormal"),
    (8192, "graphkv", "ties"),
    # beyond 327,680 tokens the tier bytes live in the scratch array itself
    (393216, "graphkv", "ties"),
    (1048576, "graphkv", "lognormal"),
])
def test_static_selection_matches_workspace_selection(T, profile, kind):
    g = torch.Generator().manual_seed(T)
    if kind == "ties":
        scores = torch.randint(0, 4, (T,), generator=g).to(torch.float32).cuda()
    else:
        scores = torch.exp(2.0 * torch.randn(T, generator=g)).cuda()
    tiers = resolve_tiers(get_profile(profile).config, T, True)
    expected = _select(False, scores, tiers)
    first = _select(True, scores, tiers)
    second = _select(True, scores, tiers)
    assert torch.equal(first, expected)
    assert torch.equal(second, expected)
    assert L.device_error() == 0


@pytest.mark.parametrize("big_T,small_T", [(65536, 12000), (1048576, 400000)])
def test_consecutive_calls_of_different_sizes(big_T, small_T):
    """The shared scratch keeps the previous call's bytes; a following smaller
    call must not see them (the second pair keeps its tier bytes in the scratch)."""
    cfg = get_profile("graphkv").config
    big = torch.randint(0, 5, (big_T,), generator=torch.Generator().manual_seed(1)).float().cuda()
    small = torch.exp(torch.randn(small_T, generator=torch.Generator().manual_seed(2))).cuda()
    t_big, t_small = resolve_tiers(cfg, big_T, True), resolve_tiers(cfg, small_T, True)
    assert torch.equal(_select(True, big, t_big), _select(False, big, t_big))
    assert torch.equal(_select(True, small, t_small), _select(False, small, t_small))
    assert L.device_error() == 0


def test_static_selection_allocates_no_device_memory():
    """What the entry point exists for: device memory in use is the same before
    and after a call (the outputs are allocated beforehand, by the caller)."""
    lib = L.lib()
    T = 131072
    scores = torch.exp(torch.randn(T, generator=torch.Generator().manual_seed(3))).cuda()
    tiers = resolve_tiers(get_profile("graphkv").config, T, True)
    idx = torch.empty(T, dtype=torch.int32, device="cuda")
    r, s, c = torch.split(idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
    pol = tiers.policy()
    st = L.stream_handle(scores.device)
    L.check(lib.gkv_select_tiers_static(scores.data_ptr(), None, ctypes.byref(pol), r.data_ptr(), s.data_ptr(),
                                        c.data_ptr(), st))  # first call: looks up the scratch address
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        L.check(lib.gkv_select_tiers_static(scores.data_ptr(), None, ctypes.byref(pol), r.data_ptr(),
                                            s.data_ptr(), c.data_ptr(), st))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert L.device_error() == 0


def test_rejects_sizes_beyond_the_scratch():
    lib = L.lib()
    T = 1048576 + 1
    pol = L.SelectPolicy(T, T, 0, 0, 0, 0, T, 0, 0, 0)
    status = lib.gkv_select_tiers_static(None, None, ctypes.byref(pol), None, None, None,
                                         L.stream_handle(torch.device("cuda")))
    assert status == L.GKV_ERR_TOO_LARGE
    assert b"exceeds" in lib.gkv_last_error()
