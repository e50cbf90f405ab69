"""gkv_mean_scores (the averaging of multi-dimensional importance scores) on the
GPU against the oracle's restatement of torch's CPU mean, bit for bit, for
shapes that take every branch of the summation order and for thread counts
beyond this host's (the column-block rule is a parameter of the call); and
against torch's own CPU mean at this host's thread counts."""
import numpy as np
import pytest
import torch

from graphkv_b200 import _lib as L
from graphkv_b200.core import _normalize_token_scores, _sum_last_block
from oracle import graphkv_oracle as orc

pytestmark = pytest.mark.gpu

SHAPES = [(2, 8192), (8, 32768), (17, 5000), (64, 1024), (64, 131072), (3, 100), (5, 7), (40, 33000),
          (100, 999), (512, 70), (1000, 33), (4096, 9), (8, 8197), (33, 8199), (1, 1)]


def _device_mean(x: np.ndarray, axis: int, threads: int) -> np.ndarray:
    t = torch.from_numpy(x).cuda()
    R, C = x.shape
    out = torch.empty(C if axis == 0 else R, dtype=torch.float32, device="cuda")
    last = _sum_last_block(R, C, threads) if axis == 0 else 0
    L.check(L.lib().gkv_mean_scores(t.data_ptr(), R, C, axis, last, out.data_ptr(),
                                    L.stream_handle(t.device)))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("threads", [1, 2, 3, 8, 24, 64, 192])
def test_kernel_matches_restated_cpu_mean(threads):
    rng = np.random.default_rng(threads)
    for R, C in SHAPES:
        x = (rng.standard_normal((R, C)) * np.exp(3.0 * rng.standard_normal((R, C)))).astype(np.float32)
        x[0, 0] = -0.0  # the output starts at +0
        for axis, xx in ((0, x), (1, np.ascontiguousarray(x.T))):
            want = (orc.torch_cpu_sum(xx, axis, threads) / np.float32(xx.shape[axis])).astype(np.float32)
            got = _device_mean(xx, axis, threads)
            assert np.array_equal(want.view(np.uint32), got.view(np.uint32)), (threads, axis, xx.shape)


def test_normalized_scores_equal_torch_cpu_mean():
    """Through the host layer, at this process's thread count: [B, T], [H, T],
    [B, H, T] and [T, X] scores give exactly torch's CPU mean."""
    g = torch.Generator().manual_seed(5)
    T = 40000
    for shape, dim in (((8, T), 0), ((3, 7, T), 0), ((T, 24), 1), ((T, 6), 1)):
        s = torch.exp(3.0 * torch.randn(*shape, generator=g))
        want = s.reshape(-1, T).mean(0) if dim == 0 else s.reshape(T, -1).mean(1)
        got = _normalize_token_scores(T, s, torch.device("cuda")).cpu()
        assert torch.equal(want.view(torch.int32), got.view(torch.int32)), shape


def test_rejects_bad_arguments():
    lib = L.lib()
    x = torch.zeros(4, 64, device="cuda")
    out = torch.empty(64, device="cuda")
    st = L.stream_handle(x.device)
    assert lib.gkv_mean_scores(x.data_ptr(), 4, 64, 2, 0, out.data_ptr(), st) == L.GKV_ERR_INVALID
    assert lib.gkv_mean_scores(x.data_ptr(), 4, 64, 0, 16, out.data_ptr(), st) == L.GKV_ERR_INVALID
    assert lib.gkv_mean_scores(None, 4, 64, 0, 0, out.data_ptr(), st) == L.GKV_ERR_INVALID
    assert lib.gkv_last_error()
