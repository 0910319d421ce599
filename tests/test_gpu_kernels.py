"""Kernel-level parity of the sm_100a path (through the C ABI) against the oracle and malkin's golden outputs."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TYPES = (8, 12, 14)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def exact_q8(monkeypatch, t=8):
    """Every GEMM keeps malkin's exact int8 block dots and per-block float order; nothing to select."""


def test_quantize_q8_bit_exact(mk, golden, torch_cuda):
    """BlockQ8 bit-identical to kern::quantize_row_q8 given the same floats (kernels_avx512.cpp:66-80)."""
    torch = torch_cuda
    x = golden["q8_x"]
    xd = dev(torch, x)
    out = torch.zeros(x.shape[0] * x.shape[1] // 32 * 40, dtype=torch.uint8, device="cuda")
    mk.quantize_q8(xd.data_ptr(), x.shape[0], x.shape[1], out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), golden["q8_blocks"].reshape(-1))


def test_quantize_i8_bit_exact(mk, golden, torch_cuda):
    torch = torch_cuda
    x = golden["i8_x"]
    q = torch.zeros(x.shape, dtype=torch.int8, device="cuda")
    d = torch.zeros(x.shape[0], dtype=torch.float32, device="cuda")
    mk.quantize_i8(dev(torch, x).data_ptr(), x.shape[0], x.shape[1], q.data_ptr(), d.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), golden["i8_q"]) and np.array_equal(d.cpu().numpy(), golden["i8_d"])


@pytest.mark.parametrize("t", TYPES)
def test_block_dots_bit_exact(mk, oracle, golden, torch_cuda, t):
    """Exact int8 block dot products (gemm_avx512.cpp:83-98, 130-141, 179-199): identical to the oracle's."""
    torch = torch_cuda
    w, x = golden[f"mm{t}_w"], golden[f"mm{t}_x"]
    W = mk.Weight(t, w, 35, 512)
    nblk = 512 // 32 * (2 if t == 14 else 1)
    out = torch.zeros((35, x.shape[0], nblk), dtype=torch.int32, device="cuda")
    W.block_dots(dev(torch, x).data_ptr(), x.shape[0], out.data_ptr())
    assert np.array_equal(out.cpu().numpy(), oracle.block_dots(t, w, 35, 512, x))


@pytest.mark.parametrize("t", TYPES)
def test_matmul_bit_exact_split1(mk, golden, torch_cuda, monkeypatch, t):
    """split_k = 1 keeps malkin's block order per (row, token): y bit-identical to its compact panel kernels."""
    exact_q8(monkeypatch, t)
    torch = torch_cuda
    w, x = golden[f"mm{t}_w"], golden[f"mm{t}_x"]
    W = mk.Weight(t, w, 35, 512)
    quantum = 16  # every type streams in 16-row panels by default (HBM bytes = GGUF bytes of the padded rows)
    assert W.device_bytes == ((35 + quantum - 1) // quantum) * quantum * mk.row_bytes(t, 512)
    y = torch.full((x.shape[0], 35), np.nan, dtype=torch.float32, device="cuda")
    W.matmul(dev(torch, x).data_ptr(), x.shape[0], y.data_ptr(), split_k=1)
    assert np.array_equal(y.cpu().numpy(), golden[f"mm{t}_y"])


@pytest.mark.parametrize("t", TYPES)
def test_matmul_split_k(mk, golden, torch_cuda, monkeypatch, t):
    """Split-K reassociates the block sum: same values within float rounding."""
    exact_q8(monkeypatch, t)
    torch = torch_cuda
    w, x = golden[f"mm{t}_w"], golden[f"mm{t}_x"]
    W = mk.Weight(t, w, 35, 512)
    ref = golden[f"mm{t}_y"]
    for split in (2, 3, 0):
        y = torch.zeros((x.shape[0], 35), dtype=torch.float32, device="cuda")
        W.matmul(dev(torch, x).data_ptr(), x.shape[0], y.data_ptr(), split_k=split)
        assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n", [1, 7, 8, 136, 150, 300])
def test_matmul_shapes_vs_oracle(mk, oracle, torch_cuda, monkeypatch, t, n):
    """Ragged rows (not a multiple of 16), token counts across the 8-token tiles and the 144-token passes."""
    exact_q8(monkeypatch, t)
    torch = torch_cuda
    from make_golden import random_rows
    rng = np.random.default_rng(n * 31 + t)
    rows, cols = 53, 1024
    w = random_rows(rng, t, rows, cols)
    x = rng.uniform(-3, 3, (n, cols)).astype(np.float32)
    W = mk.Weight(t, w, rows, cols)
    y = torch.zeros((n, rows), dtype=torch.float32, device="cuda")
    W.matmul(dev(torch, x).data_ptr(), n, y.data_ptr(), split_k=1)
    assert np.array_equal(y.cpu().numpy(), oracle.matmul(t, w, rows, cols, x))


GEMM_SHAPES = [(8, wp, ntw) for wp, lo, hi in ((8, 1, 18), (4, 4, 9), (2, 2, 5), (1, 1, 3)) for ntw in range(lo, hi + 1)]


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("wp,ntw", [(wp, ntw) for _, wp, ntw in GEMM_SHAPES])
def test_matmul_every_kernel_shape(mk, oracle, torch_cuda, monkeypatch, t, wp, ntw):
    """Every compiled shape of the panel GEMM (2 wp panels x 8 / wp x ntw token tiles per CTA, token passes over 150
    tokens), forced with MALKIN_B200_GEMM_PLAN: bit-identical to malkin's compact-panel arithmetic (the oracle)."""
    torch = torch_cuda
    from make_golden import random_rows
    monkeypatch.setenv("MALKIN_B200_GEMM_PLAN", f"{wp}:{ntw}")
    monkeypatch.setenv("MALKIN_B200_Q8_LAYOUT", "panels")
    rng = np.random.default_rng(wp * 100 + ntw + t)
    rows, cols, n = 200, 512 if t == 8 else 1024, 150
    w = random_rows(rng, t, rows, cols)
    x = rng.uniform(-3, 3, (n, cols)).astype(np.float32)
    W = mk.Weight(t, w, rows, cols)
    y = torch.full((n, rows), np.nan, dtype=torch.float32, device="cuda")
    W.matmul(dev(torch, x).data_ptr(), n, y.data_ptr(), split_k=1)
    assert np.array_equal(y.cpu().numpy(), oracle.matmul(t, w, rows, cols, x))


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n", [1, 2, 7, 17, 32, 45])
@pytest.mark.parametrize("odd", [False, True])
def test_matmul_dp4a_vs_oracle(mk, oracle, torch_cuda, monkeypatch, t, n, odd):
    """The small-row dp4a kernel (a warp per panel x 2 tokens, exact integer dots by dp4a), forced with
    MALKIN_B200_GEMM_PLAN=dp4a: ragged rows, odd token counts, a partial last tile, and k-unit counts that fill the
    last shared-memory stage or leave it part empty (odd); bit-identical to malkin's compact-panel arithmetic (the
    oracle)."""
    torch = torch_cuda
    from make_golden import random_rows
    monkeypatch.setenv("MALKIN_B200_GEMM_PLAN", "dp4a")
    monkeypatch.setenv("MALKIN_B200_Q8_LAYOUT", "panels")
    rng = np.random.default_rng(n * 13 + t + 7 * odd)
    rows = 200
    cols = (736 if odd else 768) if t == 8 else (1280 if odd else 1536)  # Q8_0: 23 / 24 blocks; K-quants: 5 / 6
    w = random_rows(rng, t, rows, cols)
    x = rng.uniform(-3, 3, (n, cols)).astype(np.float32)
    W = mk.Weight(t, w, rows, cols)
    y = torch.full((n, rows), np.nan, dtype=torch.float32, device="cuda")
    W.matmul(dev(torch, x).data_ptr(), n, y.data_ptr(), split_k=1)
    assert np.array_equal(y.cpu().numpy(), oracle.matmul(t, w, rows, cols, x))


def test_silu(mk, golden, torch_cuda):
    torch = torch_cuda
    g = dev(torch, golden["silu_g"])
    mk.silu_mul(g.data_ptr(), dev(torch, golden["silu_u"]).data_ptr(), g.numel())
    assert np.array_equal(g.cpu().numpy(), golden["silu_y"])  # malkin's exp and operation order


def _attention(mk, torch, q, H, KV, D, k, v, ks, vs, kv_base, n_keys, anc):
    """q [n, H*D]; k / v [KV, rows, D]; ks / vs [KV, rows]; anc: per token list of extra rows."""
    n = q.shape[0]
    off = np.zeros(n + 1, dtype=np.int32)
    flat = []
    for i, a in enumerate(anc):
        flat += list(a)
        off[i + 1] = len(flat)
    out = torch.zeros((n, H * D), dtype=torch.float32, device="cuda")
    tens = [dev(torch, a) for a in (q, k, v, ks, vs, np.asarray(kv_base, np.int32), np.asarray(n_keys, np.int32), off,
                                    np.asarray(flat or [0], np.int32))]
    mk.attention(tens[0].data_ptr(), n, H, KV, D, tens[1].data_ptr(), tens[2].data_ptr(), tens[3].data_ptr(),
                 tens[4].data_ptr(), k.shape[1], tens[5].data_ptr(), tens[6].data_ptr(), tens[7].data_ptr(),
                 tens[8].data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_attention_golden(mk, golden, torch_cuda):
    """Tree-masked GQA vs malkin's attend_gqa (extra ancestor keys after the prefix)."""
    torch = torch_cuda
    for i in range(4):
        G, D, n = map(int, golden[f"att{i}_shape"])
        k, v = golden[f"att{i}_k"], golden[f"att{i}_v"]
        out = _attention(mk, torch, golden[f"att{i}_q"].reshape(1, -1), G, 1, D, k[None], v[None],
                         golden[f"att{i}_ks"][None], golden[f"att{i}_vs"][None], [0], [n], [golden[f"att{i}_extra"]])
        assert np.array_equal(out.reshape(-1), golden[f"att{i}_out"])  # malkin's operation order: bit-identical


@pytest.mark.parametrize("H,KV,D", [(8, 2, 128), (16, 8, 128), (40, 8, 128), (64, 8, 128), (8, 8, 128), (24, 8, 64),
                                     (4, 2, 64), (4, 1, 256)])
def test_attention_tree_batch_vs_oracle(mk, oracle, torch_cuda, H, KV, D):
    """Two sequences, a 9-node tree on one and a 5-token prompt chunk on the other, long prefix (several key chunks
    and P.V tiles): bit-identical to the oracle's restatement of attend_gqa for G = 1, 2, 3, 4, 5, 8 and D = 64, 128, 256."""
    _tree_batch_check(mk, oracle, torch_cuda, H, KV, D)


@pytest.mark.parametrize("width", [32, 16, 8, 4])
@pytest.mark.parametrize("H,KV,D", [(8, 2, 128), (40, 8, 128), (4, 1, 256)])
def test_attention_forced_widths(mk, oracle, torch_cuda, monkeypatch, H, KV, D, width):
    """Every softmax CTA width (slots per CTA) and P.V value-slice width that the per-launch rule can pick, forced:
    each bit-identical to the oracle."""
    monkeypatch.setenv("MALKIN_B200_SM_SLOTS", str(width))
    monkeypatch.setenv("MALKIN_B200_PV_SLICE", str(width))
    _tree_batch_check(mk, oracle, torch_cuda, H, KV, D)


def _tree_batch_check(mk, oracle, torch, H, KV, D):
    rng = np.random.default_rng(5 + H + D)
    n_ctx = 700
    G = H // KV
    rows = 2 * n_ctx
    k = rng.integers(-127, 128, (KV, rows, D)).astype(np.int8)
    v = rng.integers(-127, 128, (KV, rows, D)).astype(np.int8)
    ks = rng.uniform(0.005, 0.03, (KV, rows)).astype(np.float32)
    vs = rng.uniform(0.005, 0.03, (KV, rows)).astype(np.float32)
    P = 600
    toks = []  # (kv_base, n_keys, anc)
    toks.append((0, P + 1, []))
    par = {0: []}
    for i in range(4):
        parent = 0 if i == 0 else 2 * i - 1
        for j, row in ((2 * i + 1, P + 1 + 2 * i), (2 * i + 2, P + 2 + 2 * i)):
            a = par[parent] + [row]
            par[j] = a
            toks.append((0, P + 1, a))
    for p in range(300, 305):
        toks.append((n_ctx, p + 1, []))
    n = len(toks)
    q = rng.uniform(-2, 2, (n, H * D)).astype(np.float32)
    out = _attention(mk, torch, q, H, KV, D, k, v, ks, vs, [t[0] for t in toks], [t[1] for t in toks],
                     [t[2] for t in toks])
    scale = np.float32(1.0 / np.sqrt(D))
    for t, (base, nk, anc) in enumerate(toks):
        for g in range(KV):
            want = oracle.attend(q[t, g * G * D:(g + 1) * G * D], G, D, k[g, base:], v[g, base:], ks[g, base:],
                                 vs[g, base:], nk, anc, scale)
            assert np.array_equal(out[t, g * G * D:(g + 1) * G * D], want), (t, g)


@pytest.mark.parametrize("rows,cols,n", [(128, 256, 16), (300, 512, 136), (257, 2048, 144), (130, 96, 256),
                                         (64, 512, 257), (200, 1024, 433)])
def test_q8_tensor_core_shapes_vs_oracle(mk, oracle, torch_cuda, monkeypatch, rows, cols, n):
    """Q8_0 on tcgen05 kind::i8: partial 128-row tiles, K not a multiple of the 4-block stage, N = 16 .. 256 and
    256-token passes; split 1 bit-identical to malkin's block order, and the exact block dots of the same MMAs."""
    exact_q8(monkeypatch)
    torch = torch_cuda
    from make_golden import random_rows
    rng = np.random.default_rng(rows * 7 + cols + n)
    w = random_rows(rng, 8, rows, cols)
    x = rng.uniform(-3, 3, (n, cols)).astype(np.float32)
    W = mk.Weight(8, w, rows, cols)
    y = torch.full((n, rows), np.nan, dtype=torch.float32, device="cuda")
    W.matmul(dev(torch, x).data_ptr(), n, y.data_ptr(), split_k=1)
    assert np.array_equal(y.cpu().numpy(), oracle.matmul(8, w, rows, cols, x))
    dots = torch.zeros((rows, n, cols // 32), dtype=torch.int32, device="cuda")
    W.block_dots(dev(torch, x).data_ptr(), n, dots.data_ptr())
    assert np.array_equal(dots.cpu().numpy(), oracle.block_dots(8, w, rows, cols, x))
    for split in (2, 5, 0):
        y.fill_(np.nan)
        W.matmul(dev(torch, x).data_ptr(), n, y.data_ptr(), split_k=split)
        ref = oracle.matmul(8, w, rows, cols, x)
        assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


def test_q8_layouts_agree(mk, golden, torch_cuda, monkeypatch):
    """The mma.sync panel kernel (MALKIN_B200_Q8_LAYOUT=panels) and the tcgen05 kernel give identical bits."""
    torch = torch_cuda
    w, x = golden["mm8_w"], golden["mm8_x"]
    ys = []
    exact_q8(monkeypatch)
    for layout in ("panels", "tc"):
        monkeypatch.setenv("MALKIN_B200_Q8_LAYOUT", layout)
        W = mk.Weight(8, w, 35, 512)
        y = torch.zeros((x.shape[0], 35), dtype=torch.float32, device="cuda")
        W.matmul(dev(torch, x).data_ptr(), x.shape[0], y.data_ptr(), split_k=1)
        ys.append(y.cpu().numpy())
    assert np.array_equal(ys[0], ys[1]) and np.array_equal(ys[0], golden["mm8_y"])
