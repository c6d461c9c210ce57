"""dfc_mt_step through the C ABI against the oracle, bit for bit, on seeded
random inputs: every moment format, FP32 and bf16 gradients, ragged and
misaligned segments, several hyper sets, the multi-launch batching, special
values, and the device-side gradient scale."""

import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from t3st_b200 import _lib, kernels

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 2, 3, 4, 5, 7, 8, 31, 4095, 4096, 4097, 8191, 12291, 65537, 300001]


def _rows(k):
    out = []
    for j in range(k):
        lr = [1e-3, 3e-4, 2e-2][j % 3]
        betas = [(0.9, 0.999), (0.8, 0.95), (0.5, 0.9999)][j % 3]
        wd = [0.01, 0.0, 0.1][j % 3]
        eps = [1e-8, 1e-6, 1e-12][j % 3]
        step = 1 + 7 * j
        h = O.reference_hyper(lr, betas, eps, wd, step)
        out.append(h)
    return out


def _row_tuple(h):
    return (h.beta1, h.one_minus_beta1, h.beta2, h.one_minus_beta2, h.sqrt_bc2, h.eps, h.decay,
            h.neg_step_size, h.grad_scale)


def _make_inputs(rng, n, mode, bf16, specials=False):
    p = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g = (rng.standard_t(3, n) * 1e-3).astype(np.float32)
    g[rng.random(n) < 0.05] = 0.0
    den = rng.random(n) < 0.01
    g[den] = (rng.integers(1, 1 << 23, n, dtype=np.uint32) | (rng.integers(0, 2, n, dtype=np.uint32) << 31)).view(np.float32)[den]
    if specials and n >= 8:
        g[:4] = [np.inf, -np.inf, np.nan, 3.0e38]
        p[4] = np.nan
    m = (rng.standard_normal(n) * 1e-4).astype(np.float32).view(np.uint32)
    v = (np.abs(rng.standard_normal(n)) * 1e-7).astype(np.float32).view(np.uint32)
    if mode != O.MODE_PLAIN:
        v = v | (rng.integers(0, 2, n, dtype=np.uint32) << 31)
    if mode == O.MODE_PACKED:
        m = (m & np.uint32(0xFFFF0000)) | rng.integers(0, 1 << 16, n, dtype=np.uint32)
        v = (v & np.uint32(0xFFFF0000)) | rng.integers(0, 1 << 16, n, dtype=np.uint32)
    if bf16:
        gb = (g.view(np.uint32) >> 16).astype(np.uint16)
        return p, gb, m, v
    return p, g, m, v


def _same(a, b):
    """Bit equality, with every NaN equal to every NaN (the GPU's NaN
    pattern is canonical, the CPU propagates the input's)."""
    a = np.asarray(a).view(np.uint32)
    b = np.asarray(b).view(np.uint32)
    fa = a.view(np.float32)
    fb = b.view(np.float32)
    both_nan = np.isnan(fa) & np.isnan(fb)
    return np.all((a == b) | both_nan)


def _run_case(dev, sizes, mode, bf16, n_hypers, offset_elems, seed, specials=False, scale=None):
    rng = np.random.default_rng(seed)
    hs = _rows(n_hypers)
    host, dev_tensors = [], []
    for k, n in enumerate(sizes):
        p, g, m, v = _make_inputs(rng, n, mode, bf16, specials)
        off = offset_elems[k % len(offset_elems)]
        def put(a, dt):
            buf = torch.zeros(n + off + 4, dtype=dt, device=dev)
            t = buf[off:off + n]
            t.copy_(torch.from_numpy(a.view({torch.float32: np.float32, torch.int32: np.int32, torch.int16: np.int16}[dt])))
            return t
        tp = put(p, torch.float32)
        tg = put(g.view(np.int16), torch.int16) if bf16 else put(g, torch.float32)
        if bf16:
            tg = tg.view(torch.bfloat16)
        tm = put(m.view(np.int32), torch.int32)
        tv = put(v.view(np.int32), torch.int32)
        host.append((p, g, m, v, k % n_hypers))
        dev_tensors.append((tp, tg, tm, tv))
    segs = np.zeros(len(sizes), dtype=_lib.SEGMENT_DTYPE)
    for k, (tp, tg, tm, tv) in enumerate(dev_tensors):
        segs[k] = (tp.data_ptr(), tg.data_ptr(), tm.data_ptr(), tv.data_ptr(), sizes[k],
                   k % n_hypers, _lib.GRAD_BF16 if bf16 else _lib.GRAD_F32, _lib.DTYPE_F32)
    hyp = kernels.hypers([_row_tuple(h) for h in hs])
    dscale = None
    if scale is not None:
        dscale = torch.tensor([scale], dtype=torch.float32, device=dev)
    kernels.mt_step_raw(segs, hyp, mode, dev, dscale)
    torch.cuda.synchronize()
    for k, (p, g, m, v, hi) in enumerate(host):
        h = hs[hi]
        if scale is not None:
            # the kernel applies (g * grad_scale) * scale; grad_scale is 1 here
            h = O.Hyper(**{**h.__dict__, "grad_scale": float(np.float32(scale))})
        O.step(mode, h, p, g, m, v)
        tp, tg, tm, tv = dev_tensors[k]
        assert _same(tp.cpu().numpy(), p), (k, sizes[k])
        assert _same(tm.cpu().numpy().view(np.uint32), m), (k, sizes[k])
        assert _same(tv.cpu().numpy().view(np.uint32), v), (k, sizes[k])
        if mode != O.MODE_PLAIN:
            np.testing.assert_array_equal(tv.cpu().numpy().view(np.uint32) >> 31, v >> 31)


@pytest.mark.parametrize("mode", [O.MODE_PLAIN, O.MODE_SIGNFIBER, O.MODE_PACKED])
@pytest.mark.parametrize("bf16", [False, True])
def test_ragged_aligned(cuda, mode, bf16):
    _run_case(cuda, SIZES, mode, bf16, n_hypers=3, offset_elems=[0], seed=10 + mode)


@pytest.mark.parametrize("mode", [O.MODE_SIGNFIBER, O.MODE_PACKED])
def test_misaligned_segments_take_the_scalar_path(cuda, mode):
    _run_case(cuda, SIZES, mode, False, n_hypers=2, offset_elems=[1, 2, 3, 0], seed=20 + mode)


def test_bf16_misaligned(cuda):
    _run_case(cuda, SIZES, O.MODE_PACKED, True, n_hypers=2, offset_elems=[1, 3], seed=31)


@pytest.mark.parametrize("mode", [O.MODE_PLAIN, O.MODE_SIGNFIBER, O.MODE_PACKED])
def test_special_values(cuda, mode):
    _run_case(cuda, [4096, 4103, 9], mode, False, n_hypers=1, offset_elems=[0], seed=40 + mode,
              specials=True)


def test_many_segments_and_hyper_sets_split_into_launches(cuda):
    rng = np.random.default_rng(5)
    sizes = [int(s) for s in rng.integers(1, 700, 1300)]
    _run_case(cuda, sizes, O.MODE_PACKED, False, n_hypers=40, offset_elems=[0, 1], seed=50)


def test_device_grad_scale(cuda):
    _run_case(cuda, [5000, 77], O.MODE_SIGNFIBER, False, n_hypers=1, offset_elems=[0], seed=60,
              scale=0.37)


def test_pack_unpack_kernels_match_oracle(cuda):
    rng = np.random.default_rng(6)
    n = 100003
    x = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    t = torch.from_numpy(x.view(np.int32)).to(cuda)
    kernels.pack_moments(t, second=False)
    want = O.pack_first(x.view(np.float32))
    np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32), want)
    kernels.unpack_moments(t, second=True)
    np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32), O.unpack_second(want))


def test_errors_surface_as_exceptions(cuda):
    p = torch.zeros(17, device=cuda)
    g = torch.zeros(17, device=cuda)
    m = torch.zeros(17, dtype=torch.int32, device=cuda)
    v = torch.zeros(17, dtype=torch.int32, device=cuda)
    segs = kernels.segments([p], [g], [m], [v], [0])
    segs["param"][0] += 2  # not 4-byte aligned
    hyp = kernels.hypers([_row_tuple(O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.0, 1))])
    with pytest.raises(_lib.DfcError, match="aligned"):
        kernels.mt_step_raw(segs, hyp, O.MODE_SIGNFIBER, cuda)
    segs["param"][0] -= 2
    segs["hyper"][0] = 3
    with pytest.raises(_lib.DfcError, match="hyper"):
        kernels.mt_step_raw(segs, hyp, O.MODE_SIGNFIBER, cuda)
    assert torch.count_nonzero(p) == 0  # nothing ran


def test_public_step_fast_path_follows_storage_and_grad_changes(cuda):
    """The steady-state fast path must notice re-pointed parameters, new
    gradient tensors, missing gradients and diverging step counters."""
    from t3st_b200 import DFCAdamW

    rng = np.random.default_rng(77)
    sizes = [1000, 37, 4096]
    p0 = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in sizes]
    params = [torch.nn.Parameter(torch.from_numpy(x.copy()).to(cuda)) for x in p0]
    opt = DFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed")
    ref = [dict(p=x.copy(), m=np.zeros(x.size, np.uint32), v=np.zeros(x.size, np.uint32)) for x in p0]
    steps = [0, 0, 0]
    group = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    fixed = [torch.zeros(n, device=cuda) for n in sizes]
    for t in range(12):
        gs = [(rng.standard_normal(n) * 1e-3).astype(np.float32) for n in sizes]
        if t < 4:  # same grad tensors every step (fast path by identity)
            for f, g in zip(fixed, gs):
                f.copy_(torch.from_numpy(g))
            for p, f in zip(params, fixed):
                p.grad = f
        else:      # new grad tensors every step
            for p, g in zip(params, gs):
                p.grad = torch.from_numpy(g).to(cuda)
        if t == 6:  # re-point a parameter's storage
            params[0].data = params[0].data.clone()
        if t == 8:
            params[1].grad = None
            gs[1] = None
        opt.step()
        O.multi_tensor_step(O.MODE_PACKED, ref, gs, group, steps)
    torch.cuda.synchronize()
    for p, r in zip(params, ref):
        np.testing.assert_array_equal(p.detach().cpu().numpy().view(np.uint32), r["p"].view(np.uint32))
    for p, r in zip(params, ref):
        np.testing.assert_array_equal(opt.state[p]["exp_avg"].cpu().numpy().view(np.uint32), r["m"])
        np.testing.assert_array_equal(opt.state[p]["exp_avg_sq"].cpu().numpy().view(np.uint32), r["v"])
    assert [opt.state[p]["step"] for p in params] == steps == [12, 11, 12]


NPDT = {"f32": (np.float32, torch.float32), "bf16": (np.uint16, torch.bfloat16),
        "f16": (np.uint16, torch.float16)}


def _lowp_bits(x, dt):
    if dt == "f32":
        return x.astype(np.float32)
    t = torch.from_numpy(x.astype(np.float32)).to(NPDT[dt][1])
    return t.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("pdt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("gdt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("mode", [O.MODE_SIGNFIBER, O.MODE_PACKED])
def test_parameter_and_gradient_types(cuda, pdt, gdt, mode):
    """Every (gradient type, parameter type) pair against the oracle, bit for
    bit, aligned and misaligned, with several sizes in one call."""
    rng = np.random.default_rng(zlib.crc32(f"{pdt}{gdt}{mode}".encode()))
    sizes = [1, 3, 4099, 1024, 33, 70000]
    h = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 4)
    host, keep = [], []
    segs = np.zeros(len(sizes), dtype=_lib.SEGMENT_DTYPE)
    codes = {"f32": _lib.DTYPE_F32, "bf16": _lib.DTYPE_BF16, "f16": _lib.DTYPE_F16}
    for k, n in enumerate(sizes):
        off = k % 3
        p = _lowp_bits(rng.standard_normal(n) * 0.02, pdt)
        g = _lowp_bits(rng.standard_normal(n) * 1e-3, gdt)
        m = (rng.standard_normal(n) * 1e-4).astype(np.float32).view(np.uint32)
        v = (np.abs(rng.standard_normal(n)) * 1e-7).astype(np.float32).view(np.uint32)
        v |= rng.integers(0, 2, n, dtype=np.uint32) << 31
        if mode == O.MODE_PACKED:
            m = O.pack_first(m.view(np.float32))
            v = O.pack_second(v)

        def put(a, tdt):
            buf = torch.zeros(n + off + 8, dtype=tdt, device=cuda)
            t = buf[off:off + n]
            src = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy())
            t.view(src.dtype).copy_(src)
            return t

        tp = put(p, NPDT[pdt][1])
        tg = put(g, NPDT[gdt][1])
        tm = put(m.view(np.int32), torch.int32)
        tv = put(v.view(np.int32), torch.int32)
        keep.append((tp, tg, tm, tv))
        host.append((p.copy(), g, m.copy(), v.copy()))
        segs[k] = (tp.data_ptr(), tg.data_ptr(), tm.data_ptr(), tv.data_ptr(), n, 0, codes[gdt],
                   codes[pdt])
    kernels.mt_step_raw(segs, kernels.hypers([_row_tuple(h)]), mode, cuda)
    torch.cuda.synchronize()
    for (p, g, m, v), (tp, tg, tm, tv) in zip(host, keep):
        O.step(mode, h, p, g, m, v, param_dtype=pdt, grad_dtype=gdt)
        got_p = tp.cpu().view(torch.int16).numpy().view(np.uint16) if pdt != "f32" else tp.cpu().numpy()
        np.testing.assert_array_equal(got_p.view(p.dtype), p)
        np.testing.assert_array_equal(tm.cpu().numpy().view(np.uint32), m)
        np.testing.assert_array_equal(tv.cpu().numpy().view(np.uint32), v)


@pytest.mark.parametrize("pdt", ["bf16", "f16"])
@pytest.mark.parametrize("mode", [O.MODE_SIGNFIBER, O.MODE_PACKED])
def test_every_16bit_parameter_pattern(cuda, pdt, mode):
    """Every 16-bit parameter bit pattern (normals, subnormals, +-0, +-Inf,
    NaNs), four times each, against gradients spread over a wide range of
    exponents (with zeros, Inf and NaN mixed in), a decay that is not a power
    of two and a large step size, so that the roundings to the parameter type
    -- of p * decay, of m, of the denominator and of the new parameter --
    meet subnormal, overflowing and NaN results; bit for bit against the
    oracle (round to nearest even, canonical NaN as PyTorch's CPU
    conversions give)."""
    rng = np.random.default_rng(100 + mode + (pdt == "f16"))
    p = np.tile(np.arange(65536, dtype=np.uint32).astype(np.uint16), 4)
    n = p.size
    sign = rng.integers(0, 2, n, dtype=np.uint32) << 31
    expo = rng.integers(0x30, 0x4C, n, dtype=np.uint32) << 23
    g = (sign | expo | rng.integers(0, 1 << 23, n, dtype=np.uint32)).view(np.float32)
    g[rng.integers(0, n, 64)] = 0.0
    g[rng.integers(0, n, 16)] = np.inf
    g[rng.integers(0, n, 16)] = np.nan
    m = (rng.standard_normal(n) * 1e-2).astype(np.float32).view(np.uint32)
    v = (np.abs(rng.standard_normal(n)) * 1e-3).astype(np.float32).view(np.uint32)
    v |= rng.integers(0, 2, n, dtype=np.uint32) << 31
    if mode == O.MODE_PACKED:
        m = O.pack_first(m.view(np.float32))
        v = O.pack_second(v)
    h = O.reference_hyper(0.5, (0.9, 0.999), 1e-8, 0.6, 3)
    tp = torch.from_numpy(p.view(np.int16).copy()).to(cuda).view(NPDT[pdt][1])
    tg = torch.from_numpy(g.copy()).to(cuda)
    tm = torch.from_numpy(m.view(np.int32).copy()).to(cuda)
    tv = torch.from_numpy(v.view(np.int32).copy()).to(cuda)
    codes = {"bf16": _lib.DTYPE_BF16, "f16": _lib.DTYPE_F16}
    segs = np.zeros(1, dtype=_lib.SEGMENT_DTYPE)
    segs[0] = (tp.data_ptr(), tg.data_ptr(), tm.data_ptr(), tv.data_ptr(), n, 0, _lib.DTYPE_F32,
               codes[pdt])
    kernels.mt_step_raw(segs, kernels.hypers([_row_tuple(h)]), mode, cuda)
    torch.cuda.synchronize()
    O.step(mode, h, p, g, m, v, param_dtype=pdt, grad_dtype="f32")
    # parameters: bit for bit, NaNs canonical
    np.testing.assert_array_equal(tp.cpu().view(torch.int16).numpy().view(np.uint16), p)
    got_m = tm.cpu().numpy().view(np.uint32)
    got_v = tv.cpu().numpy().view(np.uint32)
    if mode == O.MODE_PACKED:  # packed words store the canonical NaN: bit for bit
        np.testing.assert_array_equal(got_m, m)
        np.testing.assert_array_equal(got_v, v)
    else:  # FP32 words keep the arithmetic's NaN, whose payload differs by machine
        assert _same(got_m, m)
        assert _same(got_v & 0x7FFFFFFF, v & 0x7FFFFFFF)
        np.testing.assert_array_equal(got_v >> 31, v >> 31)  # payload bits
