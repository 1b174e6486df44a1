"""Per-kernel parity on the B200 through the C-ABI (ov_kernels.h).

Float kernels are compared with float64/float32 torch references of the
same op on the same inputs (tolerances stated per test); integer work
(argmax, position choice, scatter) is compared bit for bit with the CPU
oracle."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import check_argmax_exact  # noqa: E402
from omnivoice_b200 import _native as N  # noqa: E402

pytestmark = pytest.mark.gpu


def stream():
    return torch.cuda.current_stream().cuda_stream


def p(t):
    return t.data_ptr()


def ok(status):
    if status != 0:
        raise AssertionError(N.last_error())


def half_ulp(x):
    """One float16 ulp at |x| (absolute)."""
    a = np.maximum(np.abs(x), 6.1e-5)
    return 2.0 ** (np.floor(np.log2(a)) - 10)


def device_errors():
    flags = ctypes.c_uint32()
    ok(N.lib().ov_take_device_errors(ctypes.byref(flags), stream()))
    return flags.value


@pytest.fixture(autouse=True)
def _gpu(cuda_device, native):
    yield
    torch.cuda.synchronize()
    assert device_errors() == 0


# ------------------------------------------------------------ elementwise

@pytest.mark.parametrize("rows,width", [(1, 1024), (37, 1024), (620, 1024), (300, 256)])
def test_embed_and_norm(rows, width):
    g = torch.Generator().manual_seed(rows)
    vocab, C, V = 500, 8, 1025
    text = torch.randn(vocab, width, generator=g) * 0.02
    audio = torch.randn(C * V, width, generator=g) * 0.02
    ids = torch.randint(0, V, (C, rows), generator=g, dtype=torch.int32)
    row_text = torch.full((rows,), -1, dtype=torch.int32)
    n_text = rows // 3
    row_text[:n_text] = torch.randint(0, vocab, (n_text,), generator=g, dtype=torch.int32)
    w = 1.0 + 0.1 * torch.randn(width, generator=g)
    dev = [t.cuda() for t in (text, audio, ids, row_text, w)]
    hidden = torch.empty(rows, width, device="cuda")
    normed = torch.empty(rows, width, device="cuda", dtype=torch.float16)
    ok(N.lib().ov_embed(p(dev[0]), vocab, p(dev[3]), p(dev[1]), V, p(dev[2]), C, rows, width,
                        p(hidden), p(dev[4]), 1e-6, p(normed), stream()))
    torch.cuda.synchronize()
    want = torch.zeros(rows, width)
    for r in range(rows):
        if row_text[r] >= 0:
            want[r] = text[row_text[r]]
        else:
            acc = torch.zeros(width)
            for c in range(C):
                acc = acc + audio[c * V + ids[c, r]]
            want[r] = acc
    # Sequential float32 codebook sums in the reference's order: bit exact.
    assert torch.equal(hidden.cpu(), want)
    x = want.double()
    ref = (w.double() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6))).numpy()
    got = normed.cpu().double().numpy()
    assert (np.abs(got - ref) <= half_ulp(ref)).all()


@pytest.mark.parametrize("rows,width", [(5, 1024), (500, 1024), (33, 2048)])
def test_rmsnorm_and_gather(rows, width):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(rows, width, generator=g)
    w = 1.0 + 0.1 * torch.randn(width, generator=g)
    xd, wd = x.cuda(), w.cuda()
    out = torch.empty(rows, width, device="cuda", dtype=torch.float16)
    ok(N.lib().ov_rmsnorm(p(xd), p(wd), p(out), rows, width, 1e-6, stream()))
    idx = torch.randint(0, rows, (7,), generator=g, dtype=torch.int32)
    idxd = idx.cuda()
    out2 = torch.empty(7, width, device="cuda", dtype=torch.float16)
    ok(N.lib().ov_gather_rmsnorm(p(xd), p(idxd), 7, p(wd), p(out2), width, 1e-6, stream()))
    torch.cuda.synchronize()
    xd64 = x.double()
    ref = (w.double() * (xd64 * torch.rsqrt(xd64.pow(2).mean(-1, keepdim=True) + 1e-6))).numpy()
    assert (np.abs(out.cpu().double().numpy() - ref) <= half_ulp(ref)).all()
    assert torch.equal(out2.cpu(), out.cpu()[idx.long()])


def rope_tables(n, d=128, theta=1e6):
    cos = np.empty((n, d // 2), np.float32)
    sin = np.empty((n, d // 2), np.float32)
    ok(N.lib().ov_rope_tables(theta, d, n, cos.ctypes.data, sin.ctypes.data))
    return torch.from_numpy(cos), torch.from_numpy(sin)


def qknorm_rope_reference(qkv, qn, kn, pos, cos, sin, heads, kv_heads, eps=1e-6):
    """float64 QkNormRope (generator_kernels.hip:102-159) without the GQA repeat."""
    rows = qkv.shape[0]
    x = qkv.double().view(rows, heads + 2 * kv_heads, 128).clone()
    out = x.clone()
    for s in range(heads + kv_heads):
        w = (qn if s < heads else kn).double()
        v = x[:, s]
        v = w * (v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps))
        a, b = v[:, :64], v[:, 64:]
        c, sn = cos.double()[pos.long()], sin.double()[pos.long()]
        out[:, s, :64] = a * c - b * sn
        out[:, s, 64:] = b * c + a * sn
    return out.view(rows, -1).numpy()


def test_qknorm_rope_standalone():
    g = torch.Generator().manual_seed(4)
    rows, heads, kv = 77, 16, 8
    width = (heads + 2 * kv) * 128
    qkv = torch.randn(rows, width, generator=g)
    qn = 1 + 0.1 * torch.randn(128, generator=g)
    kn = 1 + 0.1 * torch.randn(128, generator=g)
    pos = torch.randint(0, 2000, (rows,), generator=g, dtype=torch.int32)
    cos, sin = rope_tables(4096)
    out = torch.empty(rows, width, device="cuda", dtype=torch.float16)
    # Device copies stay referenced until the kernel has run.
    d = [t.cuda() for t in (qkv, qn, kn, pos, cos, sin)]
    ok(N.lib().ov_qknorm_rope(p(d[0]), width, p(d[1]), p(d[2]), p(d[3]), p(d[4]), p(d[5]), 4096,
                              rows, heads, kv, 128, 1e-6, p(out), width, stream()))
    torch.cuda.synchronize()
    ref = qknorm_rope_reference(qkv, qn, kn, pos, cos, sin, heads, kv)
    got = out.cpu().double().numpy()
    # Two half ulps, plus float32 rounding of the rotation's O(1) terms for
    # outputs that cancel towards zero.
    assert (np.abs(got - ref) <= 2 * half_ulp(ref) + 1e-5).all()


def test_swiglu_standalone():
    g = torch.Generator().manual_seed(5)
    rows, width = 50, 3072
    gu = torch.randn(rows, 2 * width, generator=g) * 3
    out = torch.empty(rows, width, device="cuda", dtype=torch.float16)
    gud = gu.cuda()
    ok(N.lib().ov_swiglu(p(gud), rows, width, p(out), stream()))
    torch.cuda.synchronize()
    gd = gu.double()
    ref = (gd[:, :width] / (1 + torch.exp(-gd[:, :width])) * gd[:, width:]).numpy()
    assert (np.abs(out.cpu().double().numpy() - ref) <= half_ulp(ref)).all()


# ----------------------------------------------------------------- GEMM

def gemm(x, w, y, epi, args=None, workspace=None):
    M, K = x.shape
    N_ = w.shape[0]
    ws, wsb = (p(workspace), workspace.numel()) if workspace is not None else (None, 0)
    ok(N.lib().ov_gemm_f16(p(x), K, p(w), p(y), y.shape[1], M, K, N_, epi,
                           ctypes.byref(args) if args is not None else None, ws, wsb, stream()))


@pytest.mark.parametrize("M,N_,K", [(1, 128, 64), (100, 1024, 1024), (128, 4096, 1024),
                                    (240, 8200, 1024), (620, 6144, 1024), (700, 1024, 3072),
                                    (2175, 4096, 1024)])
def test_gemm_store_matches_fp64(M, N_, K):
    g = torch.Generator().manual_seed(M + N_ + K)
    x = (torch.randn(M, K, generator=g)).half()
    w = (torch.randn(N_, K, generator=g) * 0.02).half()
    y = torch.full((M, N_), float("nan"), device="cuda")
    gemm(x.cuda(), w.cuda(), y, N.OV_EPI_STORE_F32)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().T
    err = (y.cpu().double() - ref).abs()
    # float32 accumulation of K products: |error| <= K * 2^-23 * sum|x w|.
    bound = K * 2.0 ** -23 * (x.double().abs() @ w.double().abs().T) + 1e-6
    assert torch.isfinite(y).all()
    assert (err <= bound).all(), float(err.max())


@pytest.mark.parametrize("M,K", [(240, 2048), (620, 3072), (1080, 2048), (5000, 3072)])
def test_gemm_residual_split_k_is_deterministic(M, K):
    g = torch.Generator().manual_seed(K)
    N_ = 1024
    x = torch.randn(M, K, generator=g).half().cuda()
    w = (torch.randn(N_, K, generator=g) * 0.02).half().cuda()
    base = torch.randn(M, N_, generator=g).cuda()
    need = N.lib().ov_gemm_workspace_bytes(M, K, N_, N.OV_EPI_ACCUM_F32)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    outs = []
    for use_ws in (False, True, True):
        y = base.clone()
        gemm(x, w, y, N.OV_EPI_ACCUM_F32, workspace=ws if use_ws else None)
        outs.append(y)
    torch.cuda.synchronize()
    ref = base.double() + x.double() @ w.double().T
    bound = K * 2.0 ** -23 * (x.double().abs() @ w.double().abs().T) + 1e-5 * base.double().abs() + 1e-6
    for y in outs:
        assert ((y.double() - ref).abs() <= bound).all()
    assert torch.equal(outs[1], outs[2])  # split-K sums in a fixed order


@pytest.mark.parametrize("tile", ["64x1", "128x1", "256x1", "64x3", "128x2", "256x4",
                                  "64c2", "128c4", "256c2", "256c8", "256p1"])
@pytest.mark.parametrize("epi", [N.OV_EPI_STORE_F32, N.OV_EPI_ACCUM_F32])
def test_gemm_every_tile_shape(monkeypatch, tile, epi):
    """Each compiled tile width, serialised split-K factor (<bn>x<splits>,
    residual add only), cluster split-K factor (<bn>c<splits>) and the
    CTA-pair kernel (256p1), forced through OV_GEMM_TILE, against float64
    on ragged M and N.  Cluster split-K runs in both of its forms: partials
    through distributed shared memory (a workspace too small for them) and
    through global memory (a workspace of ov_gemm_workspace_bytes); both
    sum in split order, so where both forms exist they agree bit for bit."""
    if epi == N.OV_EPI_STORE_F32 and "x" in tile and not tile.endswith("x1"):
        pytest.skip("serialised split-K applies to the residual epilogue only")
    monkeypatch.setenv("OV_GEMM_TILE", tile)
    g = torch.Generator().manual_seed(7)
    M, N_, K = 333, 1000, 1024
    x = torch.randn(M, K, generator=g).half().cuda()
    w = (torch.randn(N_, K, generator=g) * 0.02).half().cuda()
    base = torch.randn(M, N_, generator=g).cuda()

    def run(ws):
        y = base.clone()
        gemm(x, w, y, epi, workspace=ws)
        return y

    small = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    outs = [run(small), run(small)]
    if "c" in tile:
        need = N.lib().ov_gemm_workspace_bytes(M, K, N_, epi)
        assert need > 4096
        big = torch.full((need,), 0xFF, dtype=torch.uint8, device="cuda")
        outs += [run(big), run(big)]
    torch.cuda.synchronize()
    ref = x.double() @ w.double().T
    if epi == N.OV_EPI_ACCUM_F32:
        ref = ref + base.double()
    bound = K * 2.0 ** -23 * (x.double().abs() @ w.double().abs().T) + 1e-5 * base.double().abs() + 1e-6
    for y in outs:
        assert ((y.double() - ref).abs() <= bound).all()
    assert torch.equal(outs[0], outs[1])
    if "c" in tile:
        assert torch.equal(outs[2], outs[3])
        if tile != "256c8":  # its slices do not fit the operand ring twice: no shared-memory form
            assert torch.equal(outs[0], outs[2])


def test_gemm_order_counter_wait_times_out_and_reports(monkeypatch):
    """Failure detection without a GPU fault.  Serialised split-K adds each
    split into y behind a per-tile order counter in the caller's workspace,
    which the caller must zero before first use; every wait on it is
    bounded (2 s).  A workspace left dirty never shows the expected count:
    the waits run out, the kernel still ends and reports
    OV_DEVICE_WAIT_TIMEOUT through the device error word, and the next call
    on a zeroed workspace is exact again."""
    import time
    monkeypatch.setenv("OV_GEMM_TILE", "128x4")
    g = torch.Generator().manual_seed(3)
    M, N_, K = 200, 512, 1024
    x = torch.randn(M, K, generator=g).half().cuda()
    w = (torch.randn(N_, K, generator=g) * 0.02).half().cuda()
    base = torch.randn(M, N_, generator=g).cuda()
    need = N.lib().ov_gemm_workspace_bytes(M, K, N_, N.OV_EPI_ACCUM_F32)
    assert need > 0
    ws = torch.full((need,), 0x55, dtype=torch.uint8, device="cuda")
    assert device_errors() == 0
    y = base.clone()
    start = time.monotonic()
    gemm(x, w, y, N.OV_EPI_ACCUM_F32, workspace=ws)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - start
    assert device_errors() & N.OV_DEVICE_WAIT_TIMEOUT
    assert 1.0 < elapsed < 60.0, elapsed
    ws.zero_()
    y = base.clone()
    gemm(x, w, y, N.OV_EPI_ACCUM_F32, workspace=ws)
    torch.cuda.synchronize()
    assert device_errors() == 0
    ref = x.double().cpu() @ w.double().cpu().T + base.double().cpu()
    bound = K * 2.0 ** -23 * (x.double().abs().cpu() @ w.double().abs().cpu().T) + 1e-5 * base.double().abs().cpu() + 1e-6
    assert ((y.cpu().double() - ref).abs() <= bound).all()


@pytest.mark.parametrize("tile", [None, "256x1", "256p1"])
def test_gemm_swiglu_epilogue(monkeypatch, tile):
    if tile:
        monkeypatch.setenv("OV_GEMM_TILE", tile)
    g = torch.Generator().manual_seed(11)
    M, K, I = 333, 1024, 3072
    x = torch.randn(M, K, generator=g).half()
    gu = (torch.randn(2 * I, K, generator=g) * 0.03).half()
    inter = np.empty((2 * I, K), np.uint16)
    ok(N.lib().ov_interleave_gate_up(gu.numpy().view(np.uint16).ctypes.data, I, K,
                                     inter.ctypes.data))
    w = torch.from_numpy(inter.view(np.float16)).cuda()
    y = torch.empty(M, I, device="cuda", dtype=torch.float16)
    gemm(x.cuda(), w, y, N.OV_EPI_SWIGLU_F16)
    torch.cuda.synchronize()
    h = x.double() @ gu.double().T
    gate, up = h[:, :I], h[:, I:]
    ref = (gate / (1 + torch.exp(-gate)) * up).numpy()
    got = y.cpu().double().numpy()
    assert (np.abs(got - ref) <= half_ulp(ref) + 1e-4).all()


@pytest.mark.parametrize("tile", ["128x1", "256x1", "256p1"])
def test_gemm_qknorm_rope_epilogue_matches_standalone_math(monkeypatch, tile):
    monkeypatch.setenv("OV_GEMM_TILE", tile)
    g = torch.Generator().manual_seed(12)
    M, K, heads, kv = 300, 1024, 16, 8
    width = (heads + 2 * kv) * 128
    x = torch.randn(M, K, generator=g).half()
    w = (torch.randn(width, K, generator=g) * 0.03).half()
    qn = 1 + 0.1 * torch.randn(128, generator=g)
    kn = 1 + 0.1 * torch.randn(128, generator=g)
    pos = torch.randint(0, 1500, (M,), generator=g, dtype=torch.int32)
    cos, sin = rope_tables(2048)
    dq, dk, dp, dc, ds = qn.cuda(), kn.cuda(), pos.cuda(), cos.cuda(), sin.cuda()
    args = N.EpilogueArgs(p(dq), p(dk), p(dp), p(dc), p(ds), 2048, heads, kv, 128, 1e-6)
    y = torch.empty(M, width, device="cuda", dtype=torch.float16)
    gemm(x.cuda(), w.cuda(), y, N.OV_EPI_QKNORM_ROPE_F16, args)
    torch.cuda.synchronize()
    proj = (x.double() @ w.double().T).float()
    ref = qknorm_rope_reference(proj, qn, kn, pos, cos, sin, heads, kv)
    got = y.cpu().double().numpy()
    assert (np.abs(got - ref) <= 2 * half_ulp(ref) + 1e-5).all()


# ------------------------------------------------------------ attention

def attention_reference(qkv, bounds, heads, kv_heads):
    """float64 per-sequence attention with the reference's half rounding
    of the normalised probabilities (generator.cpp:122-172)."""
    rows = qkv.shape[0]
    q = qkv[:, :heads * 128].double().view(rows, heads, 128)
    k = qkv[:, heads * 128:(heads + kv_heads) * 128].double().view(rows, kv_heads, 128)
    v = qkv[:, (heads + kv_heads) * 128:].double().view(rows, kv_heads, 128)
    out = torch.zeros(rows, heads, 128, dtype=torch.float64)
    grp = heads // kv_heads
    for s, e in zip(bounds[:-1], bounds[1:]):
        for h in range(heads):
            sc = q[s:e, h] @ k[s:e, h // grp].T / np.sqrt(128)
            pr = torch.softmax(sc, -1).half().double()
            out[s:e, h] = pr @ v[s:e, h // grp]
    return out.view(rows, heads * 128)


@pytest.mark.parametrize("form", ["pair", "pair_t", "single"])
@pytest.mark.parametrize("lengths,growing", [([1], False), ([5, 127], False), ([128, 129], False),
                                             ([370, 250], False), ([140, 100, 705, 375], False),
                                             ([1425, 750], False), ([700, 1300], True),
                                             ([257, 384, 1000], True)])
def test_attention_varlen(monkeypatch, lengths, growing, form):
    """Every work-item form, forced through OV_ATTN_FORM / OV_ATTN_PAIR:
    tile pairs with O = P V per tile (two softmax warpgroups, one query
    tile each), tile pairs with the output transposed (pair_t: O^T =
    V^T P^T, P in shared memory), and single tiles (four softmax
    warpgroups sharing one query tile's keys)."""
    monkeypatch.setenv("OV_ATTN_FORM", "single" if form == "single" else "pair")
    if form == "pair_t":
        monkeypatch.setenv("OV_ATTN_PAIR", "t")
    g = torch.Generator().manual_seed(sum(lengths))
    heads, kv = 16, 8
    rows = sum(lengths)
    width = (heads + 2 * kv) * 128
    qkv = torch.randn(rows, width, generator=g) * 1.5
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    if growing:
        # Keys grow along each sequence: the running row maximum rises by
        # many powers of two from one key tile to the next.
        for s, e in zip(bounds[:-1], bounds[1:]):
            ramp = torch.linspace(0.2, 6.0, e - s).unsqueeze(1)
            qkv[s:e, heads * 128:(heads + kv) * 128] *= ramp
    qkv = qkv.half()
    cu = torch.tensor(bounds, dtype=torch.int32).cuda()
    out = torch.full((rows, heads * 128), float("nan"), device="cuda", dtype=torch.float16)
    qkv_d = qkv.cuda()
    ok(N.lib().ov_attention_varlen(p(qkv_d), width, rows, p(cu), len(lengths),
                                   max(lengths), heads, kv, 128, 1.0 / np.sqrt(128), p(out),
                                   heads * 128, stream()))
    torch.cuda.synchronize()
    ref = attention_reference(qkv, bounds, heads, kv)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    # P is rounded to half before (not after) normalisation: a few half ulps.
    assert err.max() < 4e-3 + 4e-3 * ref.abs().max(), float(err.max())


def _work_list(lengths, per_item):
    """The generator's attention work list: (sequence, first tile | tiles
    per item << 24), longest sequences first."""
    order = sorted(range(len(lengths)), key=lambda q: -lengths[q])
    items = []
    for q in order:
        for tile in range(0, (lengths[q] + 127) // 128, per_item):
            items += [q, tile | (per_item << 24)]
    return torch.tensor(items, dtype=torch.int32)


@pytest.mark.parametrize("form", ["pair", "pair_t", "single"])
@pytest.mark.parametrize("seed,count,lo,hi", [(0, 40, 50, 900), (1, 300, 1, 300),
                                              (2, 12, 1, 140)])
def test_attention_work_list(monkeypatch, seed, count, lo, hi, form):
    """The generator's form of the attention: a work list of query-tile
    pairs (items of one or two tiles, one or many key tiles, the last key
    tile cut at any length) or of single tiles, one CTA per (item, head).
    The transposed pair form (pair_t) runs the same list.  Against float64."""
    if form == "pair_t":
        monkeypatch.setenv("OV_ATTN_PAIR", "t")
    rng = np.random.default_rng(seed)
    lengths = [int(v) for v in rng.integers(lo, hi + 1, size=count)]
    heads, kv = 16, 8
    rows = sum(lengths)
    width = (heads + 2 * kv) * 128
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(rows, width, generator=g) * 1.5).half()
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    items = _work_list(lengths, 1 if form == "single" else 2)
    n_items = items.numel() // 2
    cu = torch.tensor(bounds, dtype=torch.int32).cuda()
    out = torch.full((rows, heads * 128), float("nan"), device="cuda", dtype=torch.float16)
    qkv_d, items_d = qkv.cuda(), items.cuda()
    ok(N.lib().ov_attention_varlen_items(p(qkv_d), width, rows, p(cu), len(lengths),
                                         max(lengths), p(items_d), n_items,
                                         1 if form == "single" else 0, heads, kv, 128,
                                         1.0 / np.sqrt(128), p(out), heads * 128, stream()))
    torch.cuda.synchronize()
    assert device_errors() == 0
    ref = attention_reference(qkv, bounds, heads, kv)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    assert err.max() < 4e-3 + 4e-3 * ref.abs().max(), float(err.max())


def test_attention_work_list_bad_sequence_is_reported():
    """A work item naming a sequence outside [0, num_seqs) is skipped and
    reported through the device error word; the valid items still run."""
    lengths = [200, 90]
    heads, kv = 16, 8
    rows = sum(lengths)
    width = (heads + 2 * kv) * 128
    g = torch.Generator().manual_seed(5)
    qkv = (torch.randn(rows, width, generator=g) * 1.5).half()
    items = torch.cat([_work_list(lengths, 2), torch.tensor([7, 0 | (2 << 24)], dtype=torch.int32)])
    cu = torch.tensor([0, 200, 290], dtype=torch.int32).cuda()
    out = torch.zeros((rows, heads * 128), device="cuda", dtype=torch.float16)
    qkv_d, items_d = qkv.cuda(), items.cuda()
    assert device_errors() == 0
    ok(N.lib().ov_attention_varlen_items(p(qkv_d), width, rows, p(cu), 2, 200, p(items_d),
                                         items.numel() // 2, 0, heads, kv, 128,
                                         1.0 / np.sqrt(128), p(out), heads * 128, stream()))
    torch.cuda.synchronize()
    assert device_errors() == N.OV_DEVICE_BAD_ARGUMENT
    ref = attention_reference(qkv, [0, 200, 290], heads, kv)
    assert (out.cpu().double() - ref).abs().max() < 4e-3 + 4e-3 * ref.abs().max()


# ------------------------------------------------------- decoding tail

def test_score_matches_oracle(oracle_lib):
    rng = np.random.default_rng(0)
    F, C, V = 250, 8, 1025
    logits = (rng.normal(0, 2.0, size=(2 * F, C * V))).astype(np.float32)
    logits[3, 5] = logits[3, 9]  # a tie inside one row
    ld = 8224
    dl = torch.zeros(2 * F, ld, device="cuda")
    dl[:, :C * V] = torch.from_numpy(logits).cuda()
    pred = torch.empty(C, F, dtype=torch.int32, device="cuda")
    conf = torch.empty(C, F, device="cuda")
    ok(N.lib().ov_score(p(dl), ld, F, C, V, 1024, 2.0, p(pred), p(conf), stream()))
    torch.cuda.synchronize()
    want_p, want_c = oracle_lib.score(logits, F)
    gp, gc = pred.cpu().numpy(), conf.cpu().numpy()
    check_argmax_exact(gp, logits, F)
    check_argmax_exact(want_p, logits, F)  # the oracle obeys the same bar
    assert np.abs(gc - want_c).max() < 1e-4
    assert (gp != 1024).all()


@pytest.mark.parametrize("frames,temperature", [(3, 0.0), (100, 5.0), (250, 5.0), (750, 5.0)])
def test_select_matches_oracle_bit_exact(oracle_lib, frames, temperature):
    rng = np.random.default_rng(frames)
    C = 8
    n = C * frames
    codes = np.full(n, 1024, np.int32)
    already = rng.random(n) < 0.3
    codes[already] = rng.integers(0, 1024, size=already.sum())
    pred = rng.integers(0, 1024, size=n).astype(np.int32)
    conf = rng.normal(-3, 1, size=n).astype(np.float32)
    conf[rng.integers(0, n, size=n // 4)] = -2.5  # many exact ties
    gumbel = oracle_lib.reference_gumbel(frames, n) if temperature > 0 else None
    count = int((codes == 1024).sum() * 0.4) + 1
    # Two utterance rows of ids: conditional tail and unconditional copy.
    L = frames + 10
    R = L + frames
    ids = torch.full((C, R), -7, dtype=torch.int32, device="cuda")
    dcodes = torch.from_numpy(codes.reshape(C, frames)).cuda()
    dwhen = torch.full((C, frames), -1, dtype=torch.int32, device="cuda")
    g_dev = torch.from_numpy(gumbel).cuda() if gumbel is not None else None
    pd, cd = torch.from_numpy(pred).cuda(), torch.from_numpy(conf).cuda()
    ok(N.lib().ov_select_positions(
        p(pd), p(cd), C, frames, count, 5.0,
        temperature, N.OV_NOISE_BUFFER if temperature > 0 else N.OV_NOISE_NONE,
        p(g_dev) if g_dev is not None else None, 0, 9, 1024, p(dcodes), p(dwhen), p(ids), R,
        L - frames, L, stream()))
    torch.cuda.synchronize()
    want, chosen = oracle_lib.select(count, pred.reshape(C, frames), conf.reshape(C, frames),
                                     codes.reshape(C, frames), temperature=temperature,
                                     gumbel=gumbel)
    got = dcodes.cpu().numpy()
    assert np.array_equal(got, want)
    when = dwhen.cpu().numpy().reshape(-1)
    assert sorted(np.nonzero(when == 9)[0].tolist()) == sorted(chosen)
    idsc = ids.cpu().numpy()
    for i in chosen:
        c, f = divmod(i, frames)
        assert idsc[c, L - frames + f] == pred[i] and idsc[c, L + f] == pred[i]
    assert (idsc == -7).sum() == C * R - 2 * len(chosen)


def test_select_device_noise_picks_only_masked_slots():
    C, frames = 8, 400
    n = C * frames
    rng = np.random.default_rng(1)
    codes = np.full(n, 1024, np.int32)
    codes[: n // 2] = 5
    pred = rng.integers(0, 1024, size=n).astype(np.int32)
    conf = rng.normal(-3, 1, size=n).astype(np.float32)
    dcodes = torch.from_numpy(codes).cuda()
    pd, cd = torch.from_numpy(pred).cuda(), torch.from_numpy(conf).cuda()
    ok(N.lib().ov_select_positions(p(pd), p(cd), C, frames, 300, 5.0, 5.0,
                                   N.OV_NOISE_DEVICE, None, 1234, 3, 1024, p(dcodes), None, None,
                                   0, 0, 0, stream()))
    torch.cuda.synchronize()
    got = dcodes.cpu().numpy()
    changed = np.nonzero(got != codes)[0]
    assert (changed >= n // 2).all()
    assert ((got[n // 2:] != 1024).sum()) == 300


# ---------------------------------------------------------------- runtime

def test_graph_capture_replays_the_captured_copies():
    """ov_graph_capture_begin / _end / ov_graph_launch (include/ov_runtime.h):
    a memset and a device copy captured on a stream replay on every launch;
    the legacy stream is refused."""
    lib = N.lib()
    s = ctypes.c_void_p()
    ok(lib.ov_stream_create(ctypes.byref(s)))
    src = torch.arange(4096, dtype=torch.float32, device="cuda")
    dst = torch.zeros(4096, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ok(lib.ov_graph_capture_begin(s))
    ok(lib.ov_memset_async(p(dst), 0, dst.numel() * 4, s))
    ok(lib.ov_memcpy_d2d_async(p(dst), p(src), 2048 * 4, s))
    graph = ctypes.c_void_p()
    ok(lib.ov_graph_capture_end(s, ctypes.byref(graph)))
    for _ in range(2):
        dst.fill_(-1.0)
        torch.cuda.synchronize()
        ok(lib.ov_graph_launch(graph, s))
        ok(lib.ov_stream_sync(s))
        assert torch.equal(dst[:2048], src[:2048]) and (dst[2048:] == 0).all()
    ok(lib.ov_graph_destroy(graph))
    ok(lib.ov_stream_destroy(s))
    assert lib.ov_graph_capture_begin(None) == N.OV_ERR_INVALID
