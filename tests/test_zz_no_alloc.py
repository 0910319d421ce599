"""mk_matmul_noalloc (fixed per-device scratch, no device allocation per call) against mk_matmul on the same
inputs. Collected last, so it also runs after every other GPU test has used the device."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _weight(mk, t, rows, cols, seed):
    from make_golden import random_rows
    rng = np.random.default_rng(seed)
    w = random_rows(rng, t, rows, cols)
    return mk.Weight(t, w, rows, cols), rng


@pytest.mark.parametrize("t", [8, 12, 14])
def test_noalloc_matches_matmul_on_consecutive_calls(mk, torch_cuda, t):
    torch = torch_cuda
    rows, cols = 300, 2048
    W, rng = _weight(mk, t, rows, cols, 1234 + t)
    # two consecutive calls of different sizes: nothing from the first call may leak into the second
    for n in (136, 37):
        x = torch.from_numpy(rng.uniform(-3, 3, (n, cols)).astype(np.float32)).cuda()
        for split in (1, 0, 3):
            ref = torch.full((n, rows), float("nan"), device="cuda")
            got = torch.full((n, rows), float("nan"), device="cuda")
            W.matmul(x.data_ptr(), n, ref.data_ptr(), split_k=split)
            W.matmul_noalloc(x.data_ptr(), n, got.data_ptr(), split_k=split)
            torch.cuda.synchronize()
            assert torch.equal(ref, got), (n, split)


def test_noalloc_rejects_activations_beyond_scratch(mk, torch_cuda):
    torch = torch_cuda
    rows, cols, n = 64, 4096, 2048  # 128 blocks x 2048 tokens x 76 B > 16 MiB
    W, _ = _weight(mk, 8, rows, cols, 7)
    x = torch.zeros((n, cols), device="cuda")
    y = torch.zeros((n, rows), device="cuda")
    with pytest.raises(mk.MalkinError, match="fixed scratch"):
        W.matmul_noalloc(x.data_ptr(), n, y.data_ptr(), split_k=1)


def test_noalloc_split_limits(mk, torch_cuda):
    torch = torch_cuda
    rows, cols, n = 4096, 4096, 256  # partial sums: 4 MiB per slice
    W, rng = _weight(mk, 8, rows, cols, 11)
    x = torch.from_numpy(rng.uniform(-3, 3, (n, cols)).astype(np.float32)).cuda()
    y = torch.zeros((n, rows), device="cuda")
    with pytest.raises(mk.MalkinError, match="split_k"):
        W.matmul_noalloc(x.data_ptr(), n, y.data_ptr(), split_k=4)
    ref = torch.zeros((n, rows), device="cuda")
    W.matmul(x.data_ptr(), n, ref.data_ptr(), split_k=1)
    W.matmul_noalloc(x.data_ptr(), n, y.data_ptr(), split_k=0)  # lowers the split until the slices fit
    torch.cuda.synchronize()
    assert (y - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()
