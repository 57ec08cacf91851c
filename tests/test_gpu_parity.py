"""GPU parity: every kernel family against the CPU oracle, through the C ABI.

Bit-exact: integer/bitwise work, max/min, argmax/argmin, gather, i32
scatter_add, casts and correctly rounded float ops.  Tolerances (stated per
test) for transcendental functions (CUDA's vs the host libm the reference's
host path calls) and for float sums (the reference leaves the order free,
docs/en/ir.md:69).  The BASELINE configs are checked at full size on every
output: cfg3 rows, cfg4 table elements (f32 against an f64 segment sum, i32
bit-exact), cfg5's 2^31-element i32 chain.
"""
import math

import numpy as np
import pytest
import torch

import ask_b200
import oracle
from ask_b200 import recipes as R
from gpu_util import (NUMPY, bf16_to_f32, empty_dev, f16_to_f32, from_dev, gen_dev, run_plan, to_dev, ulp_f32)
from kat_cases import build, load_cases

pytestmark = pytest.mark.gpu
THREADS = 16
CASES = load_cases()


def same_with_nan(a: np.ndarray, b: np.ndarray) -> bool:
    a, b = np.asarray(a), np.asarray(b)
    if a.dtype.kind == "f":
        nan = np.isnan(a)
        return bool(np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32 if a.itemsize == 4
                                                                                         else np.uint64),
                                                                        b[~nan].view(np.uint32 if b.itemsize == 4
                                                                                      else np.uint64)))
    return bool(np.array_equal(a, b))


# ---- documented known answers -----------------------------------------------------
@pytest.mark.parametrize("case", CASES, ids=[f"{i}-{c['kind']}" for i, c in enumerate(CASES)])
def test_kat_on_gpu(device, case):
    kind, rec, ins, check = build(case)
    plan_types = [o["element_type"] for o in ask_b200.Plan(rec, -1).describe()["port_map"][len(ins):]]
    outs = run_plan(rec, ins, plan_types)
    assert check(outs), f"{case} -> {outs}"


# ---- generator ------------------------------------------------------------------
@pytest.mark.parametrize("kind,p0,p1,dt", [(0, -4.0, 4.0, torch.float32), (0, 0.0, 1.0, torch.float32),
                                           (4, 0, 0, torch.int32), (5, 1.1, 1 << 20, torch.int64),
                                           (6, 1.1, 1000, torch.int32)])
def test_generator_matches_host(device, kind, p0, p1, dt):
    for offset in (0, 12345, (1 << 32) - 100):
        g = gen_dev(kind, 0xA5C4, 3, 4099, p0, p1, dt, offset).cpu().numpy()
        h = oracle.generate(kind, 0xA5C4, 3, offset, 4099, p0, p1)
        assert np.array_equal(g.view(np.uint8), h.view(np.uint8)), f"kind {kind} offset {offset}"


def test_normal_generator_close_to_host(device):
    g = gen_dev(1, 0xA5C2, 0, 100000, 0.0, 1.0, torch.float32).cpu().numpy()
    h = oracle.generate(1, 0xA5C2, 0, 0, 100000, 0.0, 1.0)
    assert np.max(np.abs(g - h)) <= 1e-6
    assert abs(float(g.mean())) < 0.02 and abs(float(g.std()) - 1.0) < 0.02


# ---- cfg1: fused elementwise ---------------------------------------------------------
def cfg1_tolerance(a, b, c):
    t0 = np.maximum(np.abs(np.exp(a.astype(np.float64)) * b), np.abs(c))
    t1 = np.maximum(np.abs(np.maximum(a, b)), np.abs(np.tanh(c.astype(np.float64))))
    return 4 * ulp_f32(t0.astype(np.float32)), 4 * ulp_f32(t1.astype(np.float32))


def check_cfg1(a, b, c, y0, y1):
    r0, r1 = oracle.cfg1(a, b, c, threads=THREADS)
    tol0, tol1 = cfg1_tolerance(a, b, c)
    for got, want, tol in ((y0, r0, tol0), (y1, r1, tol1)):
        nan = np.isnan(want)
        assert np.array_equal(nan, np.isnan(got))
        fin = ~nan & np.isfinite(want)
        assert np.array_equal(got[~nan & ~fin], want[~nan & ~fin])  # infinities exactly
        err = np.abs(got[fin].astype(np.float64) - want[fin])
        assert np.all(err <= tol[fin]), f"max err {err.max()} at {np.argmax(err - tol[fin])}"


SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 88.0, 89.0, -104.0, 1e-40, -1e-45,
                    3.4e38, 0.5, 20.0, -20.0], np.float32)


@pytest.mark.parametrize("n", [1, 3, 4, 5, 17, 255, 1000, 4099])
@pytest.mark.parametrize("offset", [0, 4])
def test_cfg1_edges_and_tails(device, n, offset):
    rng = np.random.default_rng(n)
    a = rng.choice(SPECIAL, n).astype(np.float32)
    b = rng.choice(SPECIAL, n).astype(np.float32)
    c = rng.uniform(-4, 4, n).astype(np.float32)
    c[::3] = rng.choice(SPECIAL, len(c[::3]))
    y0, y1 = run_plan(R.cfg1_step(n), [a, b, c], ["f32", "f32"], offset_bytes=offset)
    check_cfg1(a, b, c, y0, y1)


def test_cfg1_full_size(device):
    n = 4096 * 4096
    a, b, c = (gen_dev(0, 0xA5C1, s, n, -4.0, 4.0, torch.float32) for s in range(3))
    plan = ask_b200.Plan(R.cfg1_step(n), 0)
    y0, y1 = torch.empty_like(a), torch.empty_like(a)
    plan.launch([a, b, c], [y0, y1], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    check_cfg1(*(t.cpu().numpy() for t in (a, b, c, y0, y1)))


# ---- cfg2: row reductions --------------------------------------------------------------
def check_rowstats(x, rows, cols, got):
    s, mx, mn, am = got
    rs, rmx, rmn, ram = oracle.rowstats(x, rows, cols, threads=THREADS)
    assert same_with_nan(mx, rmx) and same_with_nan(mn, rmn)
    assert np.array_equal(am, ram)
    absum = np.abs(x.reshape(rows, cols).astype(np.float64)).sum(axis=1)
    ref64 = x.reshape(rows, cols).astype(np.float64).sum(axis=1)
    fin = np.isfinite(ref64)
    assert np.all(np.abs(s[fin].astype(np.float64) - ref64[fin]) <= 2.0 ** -20 * absum[fin] + 1e-30)


def test_cfg2_full_size(device):
    rows, cols = 65536, 1024
    x = gen_dev(1, 0xA5C2, 0, rows * cols, 0.0, 1.0, torch.float32)
    plan = ask_b200.Plan(R.cfg2_step(rows, cols), 0)
    outs = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(3)] + \
           [torch.empty(rows, dtype=torch.int64, device="cuda")]
    plan.launch([x], outs, None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    check_rowstats(x.cpu().numpy(), rows, cols, [o.cpu().numpy() for o in outs])


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 31), (5, 32), (7, 33), (9, 100), (64, 1024), (33, 4097),
                                       (2, 70000)])
def test_cfg2_edges(device, rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    x = rng.standard_normal(rows * cols).astype(np.float32)
    # ties, signed zeros and NaNs inside rows
    x[::7] = 2.5
    x[3::11] = -0.0
    x[5::13] = 0.0
    if rows > 2:
        x[cols * 2 + min(5, cols - 1)] = np.nan
        x[cols * 2 + cols - 1] = np.nan
    if rows > 1 and cols > 2:  # infinities without NaN: exact refold of that row's values
        x[cols + 1] = np.inf
        x[cols + 2] = -np.inf
    if rows > 4:
        x[cols * 4:cols * 5] = -0.0  # an all negative-zero row: max/min must be -0, argmax/argmin 0
    outs = run_plan(R.cfg2_step(rows, cols), [x], ["f32", "f32", "f32", "i64"])
    check_rowstats(x, rows, cols, outs)


# ---- cfg3: softmax partition -------------------------------------------------------------
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_cfg3_softmax_full_size(device, dtype):
    rows, cols = 32768, 4096
    kind = 2 if dtype == "f16" else 3
    x = gen_dev(kind, 0xA5C3, 0, rows * cols, 0.0, 2.0, torch.int16)
    steps = [ask_b200.Plan(s, 0) for s in R.cfg3_steps(dtype, rows, cols)]
    m = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    y = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream()
    steps[0].launch([x], [m], None, st)
    steps[1].launch([x, m], [s], None, st)
    steps[2].launch([x, m, s], [y], None, st)
    torch.cuda.synchronize()
    # every row against the oracle's three-step f32 pipeline
    xh = x.cpu().numpy().view(np.uint16)
    rm, rs, ry = oracle.softmax(dtype, xh, rows, cols, threads=THREADS)
    gm, gs = m.cpu().numpy(), s.cpu().numpy()
    gy = y.cpu().numpy().view(np.uint16)
    assert np.array_equal(gm, rm)
    assert np.all(np.abs(gs.astype(np.float64) - rs) <= 2.0 ** -20 * rs)
    conv = f16_to_f32 if dtype == "f16" else bf16_to_f32
    gyv, ryv = conv(gy), conv(ry)
    step = np.spacing(np.abs(ryv).astype(np.float16)).astype(np.float32) if dtype == "f16" else \
        np.abs(bf16_to_f32(ry + 1) - ryv)
    assert np.all(np.abs(gyv - ryv) <= step + 1e-45), "softmax output differs by more than 1 ulp"
    # each output row sums to ~1
    rowsum = gyv.reshape(rows, cols).astype(np.float64).sum(axis=1)
    assert np.all(np.abs(rowsum - 1.0) < 0.02)


def _softmax_check(dtype, xh, rows, cols, gm, gs, gy):
    rm, rs, ry = oracle.softmax(dtype, xh, rows, cols, threads=THREADS)
    assert same_with_nan(gm, rm)  # NaN payloads are the device's canonical NaN
    fin = np.isfinite(rs)
    assert np.array_equal(np.isnan(gs), np.isnan(rs))
    assert np.all(np.abs(gs[fin].astype(np.float64) - rs[fin]) <= 2.0 ** -20 * np.abs(rs[fin]))
    conv = f16_to_f32 if dtype == "f16" else bf16_to_f32
    gyv, ryv = conv(gy), conv(ry)
    nan = np.isnan(ryv)
    assert np.array_equal(np.isnan(gyv), nan)
    step = np.spacing(np.abs(ryv[~nan]).astype(np.float16)).astype(np.float32) if dtype == "f16" else \
        np.abs(bf16_to_f32(ry[~nan] + 1) - ryv[~nan])
    assert np.all(np.abs(gyv[~nan] - ryv[~nan]) <= step + 1e-45), "softmax output differs by more than 1 ulp"


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows,cols", [(1, 256), (37, 1024), (300, 4096), (19, 8192), (5, 32768), (130, 2304)])
def test_fused_softmax_against_oracle(device, dtype, rows, cols):
    kind = 2 if dtype == "f16" else 3
    x = gen_dev(kind, 0xA5C3, 7, rows * cols, 0.0, 3.0, torch.int16)
    xh = x.cpu().numpy().view(np.uint16).copy()
    # special rows: a NaN, +inf, -inf everywhere, all -0, a huge spread (exp underflows to 0)
    nan16, inf16, ninf16 = (0x7E00, 0x7C00, 0xFC00) if dtype == "f16" else (0x7FC0, 0x7F80, 0xFF80)
    big = 0x7BFF if dtype == "f16" else 0x7F7F
    specials = [(0, 5, nan16), (min(1, rows - 1), 3, inf16)]
    for r, c, v in specials:
        xh[r * cols + c] = v
    if rows > 4:
        xh[2 * cols:3 * cols] = ninf16
        xh[3 * cols:4 * cols] = 0x8000
        xh[4 * cols] = big
    if rows > 6:  # maxima -0 and +0 in either order: m is +0 (llvm.maximum orders -0 below +0)
        neg_one = 0xBC00 if dtype == "f16" else 0xBF80
        xh[5 * cols:7 * cols] = neg_one
        xh[5 * cols + 3], xh[5 * cols + 9] = 0x8000, 0x0000
        xh[6 * cols + 3], xh[6 * cols + 9] = 0x0000, 0x8000
    x = torch.from_numpy(xh.view(np.int16)).cuda()
    plan = ask_b200.Plan({"family": "softmax", "dtype": dtype, "rows": rows, "cols": cols}, 0)
    assert plan.describe()["kernel"] == f"softmax_rows_{dtype}"
    m = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    y = torch.empty_like(x)
    plan.launch([x], [m, s, y], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    _softmax_check(dtype, xh, rows, cols, m.cpu().numpy(), s.cpu().numpy(),
                   y.cpu().numpy().view(np.uint16).reshape(-1))


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_fused_softmax_full_size_matches_three_steps(device, dtype):
    rows, cols = 32768, 4096
    x = gen_dev(2 if dtype == "f16" else 3, 0xA5C3, 0, rows * cols, 0.0, 2.0, torch.int16)
    st = torch.cuda.current_stream()
    m3, s3 = (torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(2))
    y3 = torch.empty_like(x)
    steps = [ask_b200.Plan(r, 0) for r in R.cfg3_steps(dtype, rows, cols)]
    steps[0].launch([x], [m3], None, st)
    steps[1].launch([x, m3], [s3], None, st)
    steps[2].launch([x, m3, s3], [y3], None, st)
    m1, s1 = (torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(2))
    y1 = torch.empty_like(x)
    ask_b200.Plan({"family": "softmax", "dtype": dtype, "rows": rows, "cols": cols}, 0).launch([x], [m1, s1, y1], None, st)
    torch.cuda.synchronize()
    # the three steps run on the same row kernel as the fused plan: the same
    # arithmetic in the same order, so every output agrees bit for bit
    assert [p.describe()["kernel"] for p in steps] == [f"softmax_rows_{k}_{dtype}" for k in ("max", "sum", "norm")]
    assert torch.equal(m1.view(torch.int32), m3.view(torch.int32))
    assert torch.equal(s1.view(torch.int32), s3.view(torch.int32))
    assert torch.equal(y1, y3)


def _rows_with_specials(dtype, rows, cols, seed):
    """[rows, cols] 16-bit softmax input (bits), N(0, 3), with a NaN row, an
    infinite element, an all -inf row, an all -0 row, a huge spread and rows
    whose maximum is -0 and +0 in either order."""
    x = gen_dev(2 if dtype == "f16" else 3, 0xA5C3, seed, rows * cols, 0.0, 3.0, torch.int16)
    xh = x.cpu().numpy().view(np.uint16).copy()
    nan16, inf16, ninf16 = (0x7E00, 0x7C00, 0xFC00) if dtype == "f16" else (0x7FC0, 0x7F80, 0xFF80)
    xh[5] = nan16
    xh[min(1, rows - 1) * cols + 3] = inf16
    if rows > 6:
        xh[2 * cols:3 * cols] = ninf16
        xh[3 * cols:4 * cols] = 0x8000
        xh[4 * cols] = 0x7BFF if dtype == "f16" else 0x7F7F
        xh[5 * cols:7 * cols] = 0xBC00 if dtype == "f16" else 0xBF80
        xh[5 * cols + 3], xh[5 * cols + 9] = 0x8000, 0x0000
        xh[6 * cols + 3], xh[6 * cols + 9] = 0x0000, 0x8000
    return xh


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows,cols", [(300, 4096), (37, 1024), (5, 16384), (130, 2304), (9, 256)])
def test_softmax_steps_on_the_row_kernel(device, dtype, rows, cols):
    """The plan's three steps run on the softmax row kernel (a CTA per row):
    m bit-exact, s within 2^-20 and y within one 16-bit ulp of the oracle; m
    bit-identical to the max step forced onto the warp-row reduction.  An x
    that is not 16-byte aligned takes the warp-row reduction and the
    elementwise functor at launch, with the same m; a grid cap keeps the
    normalise on the functor."""
    xh = _rows_with_specials(dtype, rows, cols, 9)
    steps = R.cfg3_steps(dtype, rows, cols)
    row_plans = [ask_b200.Plan(s, 0) for s in steps]
    assert [p.describe()["kernel"] for p in row_plans] == [f"softmax_rows_max_{dtype}", f"softmax_rows_sum_{dtype}",
                                                           f"softmax_rows_norm_{dtype}"]
    warp_plans = [ask_b200.Plan(dict(s, strategy="warp_row"), 0) for s in steps[:2]]
    norm_functor = ask_b200.Plan(dict(steps[2], blocks_per_sm=8), 0)
    assert norm_functor.describe()["kernel"] == f"ew_softmax_norm_{dtype}"
    buf = torch.empty(rows * cols + 8, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream()

    def run(plans, x, norm, y_out):
        m = torch.empty(rows, dtype=torch.float32, device="cuda")
        s = torch.empty(rows, dtype=torch.float32, device="cuda")
        plans[0].launch([x], [m], None, st)
        plans[1].launch([x, m], [s], None, st)
        norm.launch([x, m, s], [y_out], None, st)
        torch.cuda.synchronize()
        return m.cpu().numpy(), s.cpu().numpy(), y_out.cpu().numpy().view(np.uint16).copy()

    x = torch.from_numpy(xh.view(np.int16)).cuda()
    m_row, s_row, y_row = run(row_plans, x, row_plans[2], torch.empty_like(x))
    m_warp, s_warp, y_functor = run(warp_plans, x, norm_functor, torch.empty_like(x))
    buf[1:1 + rows * cols].copy_(x)  # a 2-byte offset: not 16-byte aligned
    ybuf = torch.empty(rows * cols + 8, dtype=torch.int16, device="cuda")
    m_off, s_off, y_off = run(row_plans, buf[1:1 + rows * cols], row_plans[2], ybuf[1:1 + rows * cols])
    for m, s, y in ((m_row, s_row, y_row), (m_off, s_off, y_off), (m_warp, s_warp, y_functor)):
        _softmax_check(dtype, xh, rows, cols, m, s, y)
    assert same_with_nan(m_row, m_warp)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_softmax_max_and_sum_split_over_long_rows(device, dtype):
    """Few rows of 32768: the max and sum steps take the split reduction (CTAs
    split each row, partial records combined); rows with a NaN, an infinity,
    all -inf and all -0 against the oracle."""
    rows, cols = 7, 32768
    xh = _rows_with_specials(dtype, rows, cols, 4)
    steps = R.cfg3_steps(dtype, rows, cols)[:2]
    plans = [ask_b200.Plan(s, 0) for s in steps]
    assert [p.describe()["strategy"] for p in plans] == ["split", "split"]
    x = torch.from_numpy(xh.view(np.int16)).cuda()
    st = torch.cuda.current_stream()
    m = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    scratch = [torch.empty(max(p.scratch_bytes, 16), dtype=torch.uint8, device="cuda") for p in plans]
    plans[0].launch([x], [m], scratch[0], st)
    plans[1].launch([x, m], [s], scratch[1], st)
    torch.cuda.synchronize()
    rm, rs, _ = oracle.softmax(dtype, xh, rows, cols, threads=THREADS)
    gm, gs = m.cpu().numpy(), s.cpu().numpy()
    assert same_with_nan(gm, rm)
    assert np.array_equal(np.isnan(gs), np.isnan(rs))
    fin = np.isfinite(rs)
    assert np.all(np.abs(gs[fin].astype(np.float64) - rs[fin]) <= 2.0 ** -20 * np.abs(rs[fin]))


def _rn16(q32: np.ndarray, dtype: str) -> np.ndarray:
    """f32 -> f16/bf16 bits, round to nearest even (NaN -> a quiet NaN)."""
    if dtype == "f16":
        return q32.astype(np.float16).view(np.uint16)
    b = q32.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(q32), np.uint16(0x7FC0), r)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_softmax_steps_with_given_m_and_s(device, dtype):
    """The sum and normalise steps launched on their own, with m and s that are
    not the row's own (t above 0 or below -69, s outside [2^-100, 2^24], zero,
    negative, NaN, infinite), so that units take both the paired-exp path and
    the scalar one.  Per element: t = RN32(x + RN32(-m)), e = exp(t);
    s within 2^-20 of the f64 sum of RN32(e); y within one 16-bit ulp of
    RN16(RN32(RN32(e) / s)), NaN where it is NaN, infinities exactly."""
    rng = np.random.default_rng(11)
    rows, cols = 48, 1024
    xf = rng.normal(0.0, 3.0, rows * cols).astype(np.float32)
    if dtype == "f16":
        xh = xf.astype(np.float16).view(np.uint16)
        nan16, inf16 = 0x7E00, 0x7C00
    else:
        xh = (xf.view(np.uint32) >> 16).astype(np.uint16)
        nan16, inf16 = 0x7FC0, 0x7F80
    xh[3 * cols + 100] = nan16
    xh[4 * cols + 7] = inf16
    xv = (f16_to_f32(xh) if dtype == "f16" else bf16_to_f32(xh)).reshape(rows, cols)
    with np.errstate(invalid="ignore"):
        rmax = xv.max(axis=1)
    m = np.empty(rows, np.float32)
    for r in range(rows):
        m[r] = [rmax[r], rmax[r] - 5.0, rmax[r] + 80.0, np.nan, np.inf, -np.inf, 0.0, rmax[r] + 60.0][r % 8]
    with np.errstate(all="ignore"):
        t = (xv + (m * np.float32(-1.0))[:, None]).astype(np.float32)
        e32 = np.exp(t.astype(np.float64)).astype(np.float32)
        sref = e32.astype(np.float64).sum(axis=1)
    x = torch.from_numpy(xh.view(np.int16)).cuda()
    steps = [ask_b200.Plan(r, 0) for r in R.cfg3_steps(dtype, rows, cols)]
    st = torch.cuda.current_stream()
    s_dev = torch.empty(rows, dtype=torch.float32, device="cuda")
    steps[1].launch([x, torch.from_numpy(m).cuda()], [s_dev], None, st)
    torch.cuda.synchronize()
    gs = s_dev.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isnan(gs), np.isnan(sref))
    fin = np.isfinite(sref)
    assert np.array_equal(gs[~fin & ~np.isnan(sref)], sref[~fin & ~np.isnan(sref)])
    assert np.all(np.abs(gs[fin] - sref[fin]) <= 2.0 ** -20 * np.abs(sref[fin]))
    # s given to the normalise step: the row's own sum, then values around and outside the pair range
    s_in = sref.astype(np.float32)
    for r in range(rows):
        k = (r // 8) % 6
        s_in[r] = [s_in[r], s_in[r] * 2.0 ** 25, np.float32(1e-20), 0.0, -1.5, np.inf][k] if r % 8 < 3 else s_in[r]
    s_in[47] = np.nan
    y = torch.empty_like(x)
    steps[2].launch([x, torch.from_numpy(m).cuda(), torch.from_numpy(s_in).cuda()], [y], None, st)
    torch.cuda.synchronize()
    with np.errstate(all="ignore"):
        q32 = (e32.astype(np.float64) / s_in.astype(np.float64)[:, None]).astype(np.float32)
    ry = _rn16(q32.reshape(-1), dtype)
    gy = y.cpu().numpy().view(np.uint16)
    conv = f16_to_f32 if dtype == "f16" else bf16_to_f32
    gyv, ryv = conv(gy), conv(ry)
    nan = np.isnan(ryv)
    assert np.array_equal(np.isnan(gyv), nan)
    inf = np.isinf(ryv)
    assert np.array_equal(gyv[inf], ryv[inf])
    fin = ~nan & ~inf
    step = np.spacing(np.abs(ryv[fin]).astype(np.float16)).astype(np.float32) if dtype == "f16" else \
        np.abs(conv(ry[fin] + 1) - ryv[fin])
    bad = np.abs(gyv[fin] - ryv[fin]) > step + 1e-45
    assert not bad.any(), f"{int(bad.sum())} outputs differ by more than one 16-bit ulp"


# ---- cfg4: gather / scatter_add ---------------------------------------------------------
@pytest.mark.parametrize("itype", ["i64", "i32"])
@pytest.mark.parametrize("inner,dtype", [(256, "f32"), (3, "f32"), (8, "f16"), (5, "i64"), (64, "bool")])
def test_gather_small_with_out_of_bounds(device, itype, inner, dtype):
    rows, n = 97, 301
    rng = np.random.default_rng(inner)
    table = rng.integers(0, 255, rows * inner * np.dtype(NUMPY[dtype]).itemsize, dtype=np.uint8).view(NUMPY[dtype])
    if dtype == "bool":
        table = (table & 1).astype(np.uint8)
    idx = rng.integers(-5, rows + 5, n).astype(np.int64 if itype == "i64" else np.int32)
    idx[:4] = [0, rows - 1, -1, rows]
    (out,) = run_plan(R.gather(dtype, itype, rows, inner, n), [table, idx], [dtype])
    want = oracle.gather(table, idx, 1, rows, inner)
    assert np.array_equal(out.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("dtype,inner,outer,rows,n,itype", [
    ("f32", 64, 1, 300, 5000, "i64"),     # 256-byte rows
    ("f32", 100, 3, 77, 1001, "i32"),     # 400-byte rows, outer > 1, n not a multiple of 4
    ("i64", 48, 2, 50, 33, "i64"),        # 384-byte rows
    ("f32", 512, 1, 40, 2050, "i64"),     # 2 KiB rows
    ("f32", 1024, 1, 40, 300, "i32"),     # 4 KiB rows
    ("f16", 160, 1, 1000, 70000, "i64"),  # 320-byte rows, more rows than the grid's warps
])
def test_gather_whole_rows(device, dtype, inner, outer, rows, n, itype):
    """Gathers of 16-byte-multiple rows (the vector row kernel) at several row
    sizes, outer counts and index types: every output row equals the oracle's
    and out-of-bounds rows are zero."""
    rng = np.random.default_rng(n)
    es = np.dtype(NUMPY[dtype]).itemsize
    table = rng.integers(0, 255, outer * rows * inner * es, dtype=np.uint8).view(NUMPY[dtype])
    idx = rng.integers(-3, rows + 3, n).astype(np.int64 if itype == "i64" else np.int32)
    idx[: min(n, 4)] = [0, rows - 1, -1, rows][: min(n, 4)]
    rec = R.gather(dtype, itype, rows, inner, n, outer=outer)
    (out,) = run_plan(rec, [table, idx], [dtype])
    want = oracle.gather(table, idx, outer, rows, inner)
    assert np.array_equal(out.view(np.uint8), want.view(np.uint8))


def zipf_index(n, rows, dt=torch.int64):
    return gen_dev(5 if dt == torch.int64 else 6, 0xA5C4, 1, n, 1.1, rows, dt)


def test_cfg4_gather_full_size(device):
    rows, dim, n = 1 << 20, 256, 1 << 23
    table = gen_dev(1, 0xA5C4, 0, rows * dim, 0.0, 0.02, torch.float32)
    idx = zipf_index(n, rows)
    out = torch.empty(n * dim, dtype=torch.float32, device="cuda")
    ask_b200.Plan(R.cfg4_gather_step(rows, dim, n), 0).launch([table, idx], [out], None,
                                                              torch.cuda.current_stream())
    torch.cuda.synchronize()
    t2, o2 = table.view(rows, dim).view(torch.int32), out.view(n, dim).view(torch.int32)
    for c in range(0, n, 1 << 20):  # every row, against torch's own gather as the checker
        assert torch.equal(o2[c:c + (1 << 20)], t2[idx[c:c + (1 << 20)]]), c
    # the index distribution has the Zipf(1.1) head over 2^20 rows: row 0 receives about 12.4%
    frac0 = float((idx == 0).sum()) / n
    assert 0.11 < frac0 < 0.14


@pytest.mark.parametrize("dtype", ["i32", "f32", "i64"])
@pytest.mark.parametrize("inner", [256, 5])
def test_scatter_add_small(device, dtype, inner):
    rows, n = 61, 2000
    rng = np.random.default_rng(7 + inner)
    idx = rng.integers(-3, rows + 3, n).astype(np.int64)
    idx[:50] = 0  # hot row
    if dtype == "f32":
        base = rng.standard_normal(rows * inner).astype(np.float32)
        upd = rng.standard_normal(n * inner).astype(np.float32)
    else:
        info = np.iinfo(NUMPY[dtype])
        base = rng.integers(info.min, info.max, rows * inner, dtype=NUMPY[dtype])
        upd = rng.integers(info.min, info.max, n * inner, dtype=NUMPY[dtype])
    (out,) = run_plan(R.scatter_add(dtype, "i64", rows, inner, n), [base, idx, upd], [dtype])
    if dtype == "f32":
        ref64, abs64 = oracle.scatter_add_f64(base, idx, upd, 1, rows, inner)
        assert np.all(np.abs(out - ref64) <= 2.0 ** -20 * (abs64 + np.abs(base)) + 1e-30)
    else:
        assert np.array_equal(out, oracle.scatter_add(dtype, base, idx, upd, 1, rows, inner))


def _scatter_sorted(dtype, outer, rows, inner, n, in_place, seed, zipf=True):
    """Runs the sorted scatter path on mixed Zipf-head and uniform indices
    (with out-of-range ones) and checks it against the oracle."""
    rng = np.random.default_rng(seed)
    idx = rng.integers(-2, rows + 2, n).astype(np.int64)
    if zipf:
        head = zipf_index(n, rows).cpu().numpy()
        take = rng.random(n) < 0.5
        idx[take] = head[take]
    tdt = {"f32": torch.float32, "i32": torch.int32}[dtype]
    if dtype == "f32":
        base = rng.standard_normal(outer * rows * inner).astype(np.float32)
        upd = rng.standard_normal(outer * n * inner).astype(np.float32)
    else:
        base = rng.integers(-2 ** 31, 2 ** 31 - 1, outer * rows * inner, dtype=np.int32)
        upd = rng.integers(-2 ** 31, 2 ** 31 - 1, outer * n * inner, dtype=np.int32)
    plan = ask_b200.Plan(R.scatter_add(dtype, "i64", rows, inner, n, outer=outer), 0)
    assert plan.describe()["kernel"] == "scatter_add_sorted_rows"
    d_base = torch.from_numpy(base).cuda()
    d_out = d_base if in_place else torch.empty_like(d_base)
    scratch = torch.full((plan.scratch_bytes,), 0x5A, dtype=torch.uint8, device="cuda")
    plan.launch([d_base, torch.from_numpy(idx).cuda(), torch.from_numpy(upd).cuda()], [d_out], scratch,
                torch.cuda.current_stream())
    torch.cuda.synchronize()
    out = d_out.cpu().numpy()
    del d_base, d_out, scratch
    if dtype == "f32":
        ref64, abs64 = oracle.scatter_add_f64(base, idx, upd, outer, rows, inner)
        assert np.all(np.abs(out - ref64) <= 2.0 ** -20 * (abs64 + np.abs(base)) + 1e-30)
    else:
        assert np.array_equal(out, oracle.scatter_add("i32", base, idx, upd, outer, rows, inner))


@pytest.mark.parametrize("dtype", ["f32", "i32"])
@pytest.mark.parametrize("outer,rows,inner,n,in_place", [
    (1, 1000, 16, 50000, False),    # 64-byte rows: 4 column vectors, most lanes idle
    (1, 3000, 300, 20000, False),   # 1200-byte rows: the wide-row variant with a ragged last pass
    (3, 500, 64, 7000, False),      # outer > 1: row keys o * dim + index
    (1, 2000, 256, 60000, True),    # in place: out is base, nothing is pre-copied
    (2, 700, 32, 9000, True),
])
def test_scatter_sorted_shapes(device, dtype, outer, rows, inner, n, in_place):
    _scatter_sorted(dtype, outer, rows, inner, n, in_place, seed=rows + inner)


@pytest.mark.parametrize("rows", [(1 << 22) + 1000, (1 << 24) + 5])
def test_scatter_sorted_large_tables(device, rows):
    # past 2^22 and 2^24 rows the histogram keeps 2 and then 1 counter copies
    _scatter_sorted("i32", 1, rows, 16, 1 << 18, False, seed=11)


def test_scatter_sorted_no_valid_index(device):
    rows, inner, n = 300, 64, 5000
    idx = np.full(n, rows, np.int64)
    idx[::2] = -1
    base = np.arange(rows * inner, dtype=np.int32)
    upd = np.ones(n * inner, np.int32)
    (out,) = run_plan(R.scatter_add("i32", "i64", rows, inner, n), [base, idx, upd], ["i32"], scratch_fill=0x33)
    assert np.array_equal(out, base)


def test_cfg4_scatter_full_size(device):
    rows, dim, n = 1 << 20, 256, 1 << 23
    idx = zipf_index(n, rows)
    grad = gen_dev(1, 0xA5C4, 2, n * dim, 0.0, 1.0, torch.float32)
    base = torch.zeros(rows * dim, dtype=torch.float32, device="cuda")
    out = torch.empty_like(base)
    plan = ask_b200.Plan(R.cfg4_scatter_step(rows, dim, n), 0)
    scratch = torch.empty(max(plan.scratch_bytes, 16), dtype=torch.uint8, device="cuda")
    plan.launch([base, idx, grad], [out], scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    # every table element against an f64 segment sum of its updates
    ref = torch.zeros(rows, dim, dtype=torch.float64, device="cuda")
    mag = torch.zeros_like(ref)
    gv = grad.view(n, dim)
    for c0 in range(0, n, 1 << 20):
        g = gv[c0:c0 + (1 << 20)].double()
        ref.index_add_(0, idx[c0:c0 + (1 << 20)], g)
        mag.index_add_(0, idx[c0:c0 + (1 << 20)], g.abs())
    bad = ((out.view(rows, dim).double() - ref).abs() > 2.0 ** -20 * mag).sum().item()
    assert bad == 0, f"{bad} elements outside 2^-20 * sum|upd|"
    # rows no index hits keep the base (zeros) exactly
    hit = torch.zeros(rows, dtype=torch.bool, device="cuda")
    hit[idx] = True
    assert not out.view(rows, dim)[~hit].any()


def test_cfg4_scatter_i32_bit_exact(device):
    rows, dim, n = 1 << 14, 256, 1 << 16
    idx = zipf_index(n, rows)
    upd = gen_dev(4, 0xA5C4, 5, n * dim, 0, 0, torch.int32)
    base = gen_dev(4, 0xA5C4, 6, rows * dim, 0, 0, torch.int32)
    out = torch.empty_like(base)
    plan = ask_b200.Plan(R.cfg4_scatter_step(rows, dim, n, dtype="i32"), 0)
    assert plan.describe()["kernel"] == "scatter_add_sorted_rows"
    scratch = torch.full((max(plan.scratch_bytes, 16),), 0xA5, dtype=torch.uint8, device="cuda")  # stale contents
    plan.launch([base, idx, upd], [out], scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    want = oracle.scatter_add("i32", base.cpu().numpy(), idx.cpu().numpy(), upd.cpu().numpy(), 1, rows, dim)
    assert np.array_equal(out.cpu().numpy(), want)


def test_cfg4_scatter_i32_full_size_bit_exact(device):
    """The config's shape: [2^20, 256] i32 table, 2^23 Zipf(1.1) indices,
    full-range i32 updates (sums wrap), checked on every element."""
    rows, dim, n = 1 << 20, 256, 1 << 23
    idx = zipf_index(n, rows)
    upd = gen_dev(4, 0xA5C4, 7, n * dim, 0, 0, torch.int32)
    base = gen_dev(4, 0xA5C4, 8, rows * dim, 0, 0, torch.int32)
    out = torch.empty_like(base)
    plan = ask_b200.Plan(R.cfg4_scatter_step(rows, dim, n, dtype="i32"), 0)
    assert plan.describe()["kernel"] == "scatter_add_sorted_rows"
    scratch = torch.empty(max(plan.scratch_bytes, 16), dtype=torch.uint8, device="cuda")
    plan.launch([base, idx, upd], [out], scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    want = oracle.scatter_add("i32", base.cpu().numpy(), idx.cpu().numpy(), upd.cpu().numpy(), 1, rows, dim)
    assert np.array_equal(out.cpu().numpy(), want)


# ---- cfg5: global reduction and i32 chain ---------------------------------------------
@pytest.mark.parametrize("n", [1, 100, 4097, 1 << 20, (1 << 24) + 3])
def test_cfg5a_against_oracle(device, n):
    x = gen_dev(0, 0xA5C5, 0, n, 0.0, 1.0, torch.float32)
    if n > 10:
        x[n // 3] = 0.0  # duplicate minima: the lowest index must win
    outs = [torch.empty(1, dtype=torch.float32, device="cuda") for _ in range(2)] + \
           [torch.empty(1, dtype=torch.int64, device="cuda")]
    plan = ask_b200.Plan(R.cfg5a_step(n), 0)
    scratch = torch.full((max(plan.scratch_bytes, 16),), 0x7F, dtype=torch.uint8, device="cuda")
    plan.launch([x], outs, scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    s64, sref, mn, am = oracle.cfg5a(x.cpu().numpy(), threads=THREADS)
    gs, gm, ga = float(outs[0].item()), float(outs[1].item()), int(outs[2].item())
    assert abs(gs - s64) <= 2.0 ** -20 * s64 + 1e-30
    assert gm == mn and ga == am


@pytest.mark.parametrize("special", ["inf", "-inf", "negzero"])
def test_cfg5a_specials(device, special):
    x = np.random.default_rng(1).random(300001).astype(np.float32) + 1.0
    if special == "inf":
        x[123457] = np.inf
    elif special == "-inf":
        x[200000] = -np.inf
        x[200003] = -np.inf
    else:
        x[77777] = -0.0
        x[99999] = 0.0
    s, m, a = run_plan(R.cfg5a_step(x.size), [x], ["f32", "f32", "i64"])
    s64, _, mn, am = oracle.cfg5a(x)
    assert same_with_nan(m, np.array([mn], np.float32)) and a[0] == am
    assert (np.isinf(s[0]) and np.isinf(s64)) or abs(float(s[0]) - s64) <= 2.0 ** -20 * abs(s64)


def test_cfg5a_nan_wins_first(device):
    x = np.random.default_rng(0).random(100000).astype(np.float32)
    x[777] = np.nan
    x[70000] = np.nan
    x[5] = -1.0
    s, m, a = run_plan(R.cfg5a_step(x.size), [x], ["f32", "f32", "i64"])
    assert np.isnan(s[0]) and np.isnan(m[0]) and a[0] == 777


def test_cfg5a_full_size(device):
    n = 1 << 32
    x = gen_dev(0, 0xA5C5, 0, n, 0.0, 1.0, torch.float32)
    outs = [torch.empty(1, dtype=torch.float32, device="cuda") for _ in range(2)] + \
           [torch.empty(1, dtype=torch.int64, device="cuda")]
    plan = ask_b200.Plan(R.cfg5a_step(n), 0)
    scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
    plan.launch([x], outs, scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    total, mn, first = 0.0, math.inf, -1
    chunk = 1 << 28
    for c0 in range(0, n, chunk):
        part = x[c0:c0 + chunk]
        total += float(part.double().sum())
        pm = float(part.min())
        if pm < mn:
            mn, first = pm, c0 + int(torch.nonzero(part == pm)[0])
    assert abs(float(outs[0].item()) - total) <= 2.0 ** -20 * total
    assert float(outs[1].item()) == mn and int(outs[2].item()) == first


@pytest.mark.parametrize("n", [1, 7, 1000, 1 << 20, (1 << 22) + 5])
@pytest.mark.parametrize("offset", [0, 4])
def test_cfg5b_bit_exact(device, n, offset):
    rng = np.random.default_rng(n)
    x = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    y = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    (z,) = run_plan(R.cfg5b_step(n), [x, y], ["i32"], offset_bytes=offset)
    assert np.array_equal(z, oracle.cfg5b(x, y))


def test_cfg5b_full_size(device):
    """Every one of the 2^31 outputs, bit-exact, compared in chunks."""
    n = 1 << 31
    x = gen_dev(4, 0xA5C5, 1, n, 0, 0, torch.int32)
    y = gen_dev(4, 0xA5C5, 2, n, 0, 0, torch.int32)
    z = torch.empty_like(x)
    ask_b200.Plan(R.cfg5b_step(n), 0).launch([x, y], [z], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    chunk = 1 << 28
    for c0 in range(0, n, chunk):
        sl = slice(c0, c0 + chunk)
        want = oracle.cfg5b(x[sl].cpu().numpy(), y[sl].cpu().numpy(), threads=THREADS)
        assert np.array_equal(z[sl].cpu().numpy(), want), f"chunk at {c0}"


# ---- generic (runtime-interpreted) programs ---------------------------------------------
FLOAT_BINARY = ["add", "mul", "div", "maximum", "minimum", "floordiv", "mod"]
FLOAT_UNARY = ["abs", "floor", "ceil", "round", "sqrt"]
INT_BINARY = ["add", "mul", "floordiv", "mod", "pow", "maximum", "minimum", "bitwise_and", "bitwise_or",
              "bitwise_xor", "shift_left", "shift_right"]


def random_program(rng, dtype):
    p = R.Program()
    vals = [p.input(dtype), p.input(dtype), p.input(dtype, "scalar")]
    for _ in range(10):
        r = rng.random()
        a, b = vals[rng.integers(len(vals))], vals[rng.integers(len(vals))]
        if dtype in ("f32", "f16", "bf16"):
            if r < 0.55:
                vals.append(p.op(FLOAT_BINARY[rng.integers(len(FLOAT_BINARY))], a, b))
            elif r < 0.8:
                vals.append(p.op(FLOAT_UNARY[rng.integers(len(FLOAT_UNARY))], a))
            else:
                c = p.compare(["lt", "le", "eq", "ne", "gt", "ge"][rng.integers(6)], a, b)
                vals.append(p.select(c, a, b))
        else:
            if r < 0.8:
                vals.append(p.op(INT_BINARY[rng.integers(len(INT_BINARY))], a, b))
            else:
                vals.append(p.abs(a))
    outs = [vals[-1], vals[-3], p.cast(vals[-2], "f32" if dtype != "f32" else "i32"),
            p.compare("gt", vals[-1], vals[-4])]
    return p, outs


def random_inputs(rng, dtype, n):
    if dtype == "f32":
        x = rng.standard_normal(n).astype(np.float32) * 4
        x[::5] = rng.choice(SPECIAL, len(x[::5]))
        return x
    if dtype == "f16":
        return (rng.standard_normal(n) * 8).astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return (rng.standard_normal(n).astype(np.float32) * 8).view(np.uint32).__rshift__(16).astype(np.uint16)
    if dtype == "i32":
        x = rng.integers(-100, 100, n).astype(np.int32)
        x[::7] = rng.integers(-(2 ** 31), 2 ** 31, len(x[::7]), dtype=np.int64).astype(np.int32)
        return x
    x = rng.integers(-100, 100, n).astype(np.int64)
    x[::7] = rng.integers(-(2 ** 63), 2 ** 63 - 1, len(x[::7]), dtype=np.int64)
    return x


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16", "i32", "i64"])
@pytest.mark.parametrize("seed", range(6))
def test_generic_programs_match_oracle(device, dtype, seed):
    rng = np.random.default_rng(seed * 31 + len(dtype))
    p, outs = random_program(rng, dtype)
    n = 1031
    rec = R.elementwise(p, outs, n)
    ins = [random_inputs(rng, dtype, n), random_inputs(rng, dtype, n), random_inputs(rng, dtype, 1)]
    assert ask_b200.Plan(rec, -1).describe()["kernel"] == "ew_generic"
    got = run_plan(rec, ins, [o.dtype for o in outs])
    want = oracle.elementwise(rec, ins)
    for k, (g, w) in enumerate(zip(got, want)):
        if outs[k].dtype == "f32":
            assert same_with_nan(g, w), f"output {k}"
        elif outs[k].dtype in ("f16", "bf16"):
            conv = f16_to_f32 if outs[k].dtype == "f16" else bf16_to_f32
            assert same_with_nan(conv(g), conv(w)), f"output {k}"
        else:
            assert np.array_equal(g, w), f"output {k}"


@pytest.mark.parametrize("op", ["exp", "log", "sin", "cos", "tanh", "erf", "pow"])
def test_transcendentals_within_ulps(device, op):
    rng = np.random.default_rng(11)
    n = 50000
    x = rng.uniform(-10, 10, n).astype(np.float32)
    y = rng.uniform(-3, 3, n).astype(np.float32)
    if op in ("log",):
        x = np.abs(x) + np.float32(1e-3)
    if op == "pow":
        x = np.abs(x)
    p = R.Program()
    a, b = p.input("f32"), p.input("f32")
    r = p.op(op, a, b) if op == "pow" else p.op(op, a)
    rec = R.elementwise(p, [r], n)
    (got,) = run_plan(rec, [x, y], ["f32"])
    (want,) = oracle.elementwise(rec, [x, y])
    fin = np.isfinite(want)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    err = np.abs(got[fin].astype(np.float64) - want[fin]) / ulp_f32(want[fin])
    assert err.max() <= 4, f"{op}: {err.max()} ulp"


# ---- reductions with prologues, column reductions, generic reductions ---------------------
@pytest.mark.parametrize("outer,extent,inner", [(3, 5, 7), (1, 1000, 33), (16, 64, 4), (2, 3, 1000),
                                                (1, 4096, 513), (4, 20000, 3), (2, 777, 1025)])
def test_column_reductions(device, outer, extent, inner):
    rng = np.random.default_rng(outer + extent + inner)
    x = rng.standard_normal(outer * extent * inner).astype(np.float32)
    x[::9] = 1.5
    p = R.Program()
    v = p.input("f32")
    rec = R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin", "prod"], outer, extent, inner)
    got = run_plan(rec, [x], ["f32", "f32", "f32", "i64", "i64", "f32"])
    want = oracle.reduce(rec, [x])
    assert np.array_equal(got[1], want[1]) and np.array_equal(got[2], want[2])
    assert np.array_equal(got[3], want[3]) and np.array_equal(got[4], want[4])
    xx = x.reshape(outer, extent, inner).astype(np.float64)
    tol = 2.0 ** -20 * np.abs(xx).sum(axis=1).reshape(-1)
    assert np.all(np.abs(got[0] - xx.sum(axis=1).reshape(-1)) <= tol + 1e-30)
    # products in range (over thousands of factors they overflow or underflow,
    # where the order of the f32 multiplications decides; the bar is for the rest)
    normal = (np.abs(want[5]) > 1e-30) & (np.abs(want[5]) < 1e30)
    rel = np.abs(got[5][normal].astype(np.float64) - want[5][normal]) / np.abs(want[5][normal])
    assert np.all(rel <= 1e-5)


def test_column_chunks_keep_first_positions_and_nan(device):
    """Few columns over a long extent split the extent into chunks (partial
    records in scratch, combined in chunk order): a column of equal values,
    a NaN placed late, a column of -inf and a later duplicate of the maximum
    keep the reference's first-position and NaN-first rules across chunk
    boundaries, whatever stale bytes the scratch held."""
    outer, extent, inner = 1, 5000, 8
    p = R.Program()
    v = p.input("f32")
    rec = R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin"], outer, extent, inner)
    plan = ask_b200.Plan(rec, 0)
    assert plan.describe()["kernel"] == "reduce_column_chunks_generic" and plan.describe()["launch"]["grid"][1] > 1
    x = np.random.default_rng(1).standard_normal((extent, inner)).astype(np.float32)
    x[:, 0] = 2.0                                 # all equal: positions 0
    x[4321, 1] = np.nan; x[4400, 1] = np.nan      # the first NaN wins max, min and both positions
    x[:, 2] = -np.inf                             # argmax of an all -inf column: 0
    x[1234, 3] = 9.0; x[3999, 3] = 9.0            # the first of two maxima
    x[17, 4] = -9.0; x[4999, 4] = -9.0            # the first of two minima
    for fill in (0x00, 0xFF):
        got = run_plan(rec, [x.reshape(-1)], ["f32", "f32", "f32", "i64", "i64"], scratch_fill=fill)
        want = oracle.reduce(rec, [x.reshape(-1)])
        for k in (1, 2, 3, 4):
            assert np.array_equal(got[k], want[k], equal_nan=True), (fill, k)
        assert got[3][1] == 4321 and got[4][1] == 4321 and got[3][0] == 0 and got[3][2] == 0
        assert got[3][3] == 1234 and got[4][4] == 17
        xx = x.astype(np.float64)
        fin = np.isfinite(xx.sum(axis=0))
        assert np.all(np.abs(got[0][fin] - xx.sum(axis=0)[fin]) <= 2.0 ** -20 * np.abs(xx).sum(axis=0)[fin])


@pytest.mark.parametrize("dtype", ["i32", "i64"])
def test_column_chunks_integers_exact(device, dtype):
    outer, extent, inner = 3, 3000, 5
    p = R.Program()
    v = p.input(dtype)
    rec = R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin", "prod"], outer, extent, inner)
    assert ask_b200.Plan(rec, 0).describe()["launch"]["grid"][1] > 1
    rng = np.random.default_rng(2)
    x = rng.integers(-3, 4, outer * extent * inner).astype(NUMPY[dtype])
    got = run_plan(rec, [x], [dtype, dtype, dtype, "i64", "i64", dtype])
    want = oracle.reduce(rec, [x])
    for k in range(6):
        assert np.array_equal(got[k], want[k]), k


@pytest.mark.parametrize("dtype", ["i32", "i64", "bool"])
def test_integer_and_bool_reductions(device, dtype):
    rng = np.random.default_rng(5)
    rows, cols = 37, 301
    if dtype == "bool":
        x = (rng.random(rows * cols) < 0.01).astype(np.uint8)
        ops = ["any", "all", "max", "min", "argmax", "argmin"]
    else:
        x = rng.integers(-1000, 1000, rows * cols).astype(NUMPY[dtype])
        ops = ["sum", "prod", "max", "min", "argmax", "argmin"]
    p = R.Program()
    v = p.input(dtype)
    rec = R.reduce(p, v, ops, rows, cols)
    plan_types = [o["element_type"] for o in ask_b200.Plan(rec, -1).describe()["port_map"][1:]]
    got = run_plan(rec, [x], plan_types)
    want = oracle.reduce(rec, [x])
    for g, w, op in zip(got, want, ops):
        assert np.array_equal(g, w), op


def test_reduce_with_prologue_program(device):
    rows, cols = 50, 777
    rng = np.random.default_rng(9)
    x = rng.standard_normal(rows * cols).astype(np.float32)
    w = rng.standard_normal(rows).astype(np.float32)
    p = R.Program()
    xv, wv = p.input("f32"), p.input("f32", "outer")
    val = p.mul(p.abs(p.add(xv, wv)), p.const("f32", 0.5))
    rec = R.reduce(p, val, ["max", "argmin", "sum"], rows, cols)
    assert ask_b200.Plan(rec, -1).describe()["kernel"].endswith("generic")
    got = run_plan(rec, [x, w], ["f32", "i64", "f32"])
    want = oracle.reduce(rec, [x, w])
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    ref = np.abs(x.reshape(rows, cols).astype(np.float32) + w[:, None]) * np.float32(0.5)
    assert np.allclose(got[2], ref.astype(np.float64).sum(axis=1), rtol=1e-6)


def test_split_reduction_ignores_stale_scratch(device):
    x = np.random.default_rng(1).random(1 << 20).astype(np.float32)
    rec = R.cfg5a_step(x.size)
    a = run_plan(rec, [x], ["f32", "f32", "i64"], scratch_fill=0xFF)
    b = run_plan(rec, [x], ["f32", "f32", "i64"], scratch_fill=0x00)
    assert all(np.array_equal(p, q) for p, q in zip(a, b))  # deterministic, scratch fully overwritten


@pytest.mark.parametrize("inner", [1, 3, 4, 7, 1000, 4096])
@pytest.mark.parametrize("offset", [0, 4])
def test_elementwise_index_maps(device, inner, offset):
    rows = 37
    n = rows * inner
    rng = np.random.default_rng(inner + offset)
    p = R.Program()
    x, r, c, s = p.input("f32"), p.input("f32", "outer"), p.input("f32", "inner"), p.input("f32", "scalar")
    y = p.add(p.mul(x, r), p.mul(c, s))
    z = p.maximum(p.add(x, c), r)
    rec = R.elementwise(p, [y, z], n, inner=inner)
    ins = [rng.standard_normal(n).astype(np.float32), rng.standard_normal(rows).astype(np.float32),
           rng.standard_normal(inner).astype(np.float32), np.array([1.5], np.float32)]
    got = run_plan(rec, ins, ["f32", "f32"], offset_bytes=offset)
    want = oracle.elementwise(rec, ins)
    assert same_with_nan(got[0], want[0]) and same_with_nan(got[1], want[1])
