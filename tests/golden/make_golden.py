"""Generate the golden vectors in this folder by running the reference itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <checkout of YellowJune/T3st>

It imports ``remote/torch_fiber.py`` from the reference (YellowJune/T3st),
runs its ``DFCAdamW.step`` (:68-117) on CPU tensors with seeded inputs, and
stores inputs and outputs as ``.npz``.  Nothing at test time reads the
reference; the tests only read these files.

PyTorch's CPU ``Tensor.sqrt`` is not correctly rounded (it is off by one ulp
on about 0.7% of FP32 inputs; IEEE ``sqrtf``, and CUDA's, is exact).  Every
case is therefore run twice: once stock (``p``) and once with ``Tensor.sqrt``
replaced by the correctly rounded FP32 square root -- sqrt in double, rounded
once to FP32, which is exact for square roots since 53 >= 2*24 + 2
(``p_ieee_sqrt``).  m and v do not depend on the square root and are the
same in both runs.

Cases (all FP32):
  fiber_mt       4 tensors (4099, 31x257, 31, 1), 6 steps, payload in every
                 bit 31 of v, tensor 2 has no gradient on step 3 (per-tensor
                 step counters diverge), lr 1e-3, wd 0.01.
  plain_mt       the same inputs with enable_fiber=False.
  ragged_stress  24 tensors of sizes 1..4093 (not multiples of 4 or 8),
                 Student-t(3)*1e-3 gradients with 5% exact zeros and 0.1%
                 FP32 denormals, moments pre-seeded from packed words whose
                 16-bit residual fields span the full range, random payload,
                 wd 0 (the reference skips the decay), betas (0.8, 0.95), eps 1e-6.
  c1_small       one 2^14 tensor, 12 steps, p~N(0,0.02), g~N(0,1e-3), lr 1e-3,
                 betas (0.9,0.999), eps 1e-8, wd 0.01, random payload.
  bf16_params,   3 bf16 (or fp16) parameter tensors (1031, 300, 7) with
  f16_params     gradients of the same type, 6 steps, payload, lr 1e-3, wd 0.01;
                 p is stored as the 16-bit patterns.
  replay         the replay codec and reservoir of remote/vision_benchmark.py
                 (:74-151): 24 seeded images (on the 1/255 grid like ToTensor,
                 plus exact quantisation ties, values outside [0, 1], -0.0,
                 +-Inf and NaN), their records from CIFAR4BitCodec.encode,
                 the decoded images, corrupted records with the error each
                 raises, and a FiberReservoir over an ArrayChannel (room for
                 5 records) after 12 adds and a sample of 6 (seeded rng).
  unit_linear    the reference's own unit-test trajectory
                 (remote/test_torch_fiber.py:11-31): Linear(257,31), seed 17,
                 50 steps of MSE, lr 3e-4, wd 0.01; final params of the
                 fiber-off and fiber-on runs and the payload read back.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _flat(ts):
    return np.concatenate([t.detach().reshape(-1).numpy() for t in ts]) if ts else np.empty(0)


def run_case(tf, sizes, p0, grads, none_mask, group, fiber, m0=None, v0_bits=None, payload_bits=None):
    """Drive the reference optimizer with explicit gradients.

    grads: [steps, total] float32; none_mask: [steps, n_tensors] bool (True -> grad None).
    """
    params = []
    off = 0
    for n in sizes:
        params.append(torch.nn.Parameter(torch.from_numpy(p0[off:off + n].copy())))
        off += n
    opt = tf.DFCAdamW(params, lr=group["lr"], betas=group["betas"], eps=group["eps"],
                      weight_decay=group["weight_decay"], enable_fiber=fiber)
    off = 0
    for i, p in enumerate(params):
        n = sizes[i]
        st = opt.state[p]
        if m0 is not None:
            st["exp_avg"].copy_(torch.from_numpy(m0[off:off + n].copy()))
        if v0_bits is not None:
            st["exp_avg_sq"].view(torch.int32).copy_(
                torch.from_numpy(v0_bits[off:off + n].view(np.int32).copy()))
        off += n
    if payload_bits is not None:
        ch = tf.TorchSignFiberChannel(opt)
        ch.write_bits(0, payload_bits)
    for s in range(grads.shape[0]):
        off = 0
        for i, p in enumerate(params):
            n = sizes[i]
            if none_mask[s, i]:
                p.grad = None
            else:
                p.grad = torch.from_numpy(grads[s, off:off + n].copy())
            off += n
        opt.step()
    p_out = _flat([p.data for p in params]).astype(np.float32)
    m_out = _flat([opt.state[p]["exp_avg"] for p in params]).astype(np.float32)
    v_out = np.concatenate([opt.state[p]["exp_avg_sq"].reshape(-1).view(torch.int32).numpy()
                            for p in params]).view(np.uint32)
    steps = np.array([opt.state[p]["step"] for p in params], np.int64)
    return p_out, m_out.view(np.uint32), v_out, steps


_stock_sqrt = torch.Tensor.sqrt


def _ieee_sqrt(self):
    if self.dtype == torch.float32:
        return _stock_sqrt(self.double()).float()
    return _stock_sqrt(self)


def run_both(*args, **kwargs):
    """Run a case with the stock sqrt, then with the correctly rounded one."""
    p, m, v, st = run_case(*args, **kwargs)
    torch.Tensor.sqrt = _ieee_sqrt
    try:
        p2, m2, v2, st2 = run_case(*args, **kwargs)
    finally:
        torch.Tensor.sqrt = _stock_sqrt
    assert np.array_equal(m, m2) and np.array_equal(v, v2) and np.array_equal(st, st2)
    return p, p2, m, v, st


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def group_arrays(group):
    return dict(lr=np.float64(group["lr"]), betas=np.array(group["betas"], np.float64),
                eps=np.float64(group["eps"]), weight_decay=np.float64(group["weight_decay"]))


def case_mt(tf, fiber, name):
    rng = np.random.default_rng(1001)
    sizes = [4099, 31 * 257, 31, 1]
    total = sum(sizes)
    steps = 6
    p0 = (rng.standard_normal(total) * 0.02).astype(np.float32)
    grads = (rng.standard_normal((steps, total)) * 1e-3).astype(np.float32)
    none_mask = np.zeros((steps, len(sizes)), bool)
    none_mask[2, 2] = True
    payload = rng.integers(0, 2, total, dtype=np.uint8) if fiber else None
    group = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    p, pi, m, v, st = run_both(tf, sizes, p0, grads, none_mask, group, fiber, payload_bits=payload)
    extra = {} if payload is None else {"payload": payload}
    save(name, sizes=np.array(sizes, np.int64), p0=p0, grads=grads, none_mask=none_mask,
         fiber=np.bool_(fiber), p=p, p_ieee_sqrt=pi, m=m, v=v, steps=st, **group_arrays(group),
         **extra)


def _denormal_mix(rng, shape, scale):
    g = (rng.standard_t(3, shape) * scale).astype(np.float32)
    u = rng.random(shape)
    g[u < 0.05] = 0.0
    den = u > 0.999
    mant = rng.integers(1, 1 << 23, shape, dtype=np.uint32)
    sign = rng.integers(0, 2, shape, dtype=np.uint32) << 31
    g[den] = (mant | sign).view(np.float32)[den]
    return g


def case_ragged(tf, oracle):
    rng = np.random.default_rng(2002)
    sizes = [1, 2, 3, 5, 7, 8, 9, 15, 16, 17, 31, 33, 63, 65, 127, 129, 255, 257, 511, 513,
             1023, 1025, 2047, 4093]
    total = sum(sizes)
    steps = 4
    p0 = (rng.standard_normal(total) * 0.02).astype(np.float32)
    grads = _denormal_mix(rng, (steps, total), 1e-3)
    none_mask = np.zeros((steps, len(sizes)), bool)
    none_mask[1, 5] = True
    none_mask[3, 0] = True
    # packed moment words: high half = bf16 of a plausible moment, low half = any 16 bits
    m_val = _denormal_mix(rng, total, 1e-3)
    v_val = np.abs(_denormal_mix(rng, total, 1e-6)).astype(np.float32)
    m_hi = oracle.pack_first(m_val) & np.uint32(0xFFFF0000)
    v_hi = oracle.pack_second(v_val.view(np.uint32)) & np.uint32(0x7FFF0000)
    lo_m = rng.integers(0, 1 << 16, total, dtype=np.uint32)
    lo_v = rng.integers(0, 1 << 16, total, dtype=np.uint32)
    payload = rng.integers(0, 2, total, dtype=np.uint32)
    m_words = m_hi | lo_m
    v_words = v_hi | lo_v | (payload << 31)
    m0 = oracle.unpack_first(m_words)
    v0_bits = oracle.unpack_second(v_words)  # payload in bit 31, decoded magnitude below
    group = dict(lr=3e-4, betas=(0.8, 0.95), eps=1e-6, weight_decay=0.0)
    p, pi, m, v, st = run_both(tf, sizes, p0, grads, none_mask, group, True, m0=m0, v0_bits=v0_bits)
    save("ragged_stress", sizes=np.array(sizes, np.int64), p0=p0, grads=grads, none_mask=none_mask,
         fiber=np.bool_(True), m0=m0.view(np.uint32), v0=v0_bits, m0_words=m_words,
         v0_words=v_words, p=p, p_ieee_sqrt=pi, m=m, v=v, steps=st, **group_arrays(group))


def case_c1(tf):
    rng = np.random.default_rng(3003)
    n = 1 << 14
    steps = 12
    p0 = (rng.standard_normal(n) * 0.02).astype(np.float32)
    grads = (rng.standard_normal((steps, n)) * 1e-3).astype(np.float32)
    payload = rng.integers(0, 2, n, dtype=np.uint8)
    group = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    none_mask = np.zeros((steps, 1), bool)
    p, pi, m, v, st = run_both(tf, [n], p0, grads, none_mask, group, True, payload_bits=payload)
    save("c1_small", sizes=np.array([n], np.int64), p0=p0, grads=grads, none_mask=none_mask,
         fiber=np.bool_(True), payload=payload, p=p, p_ieee_sqrt=pi, m=m, v=v, steps=st,
         **group_arrays(group))


def case_lowp(tf, dtype, name):
    rng = np.random.default_rng(4004)
    sizes = [1031, 300, 7]
    total = sum(sizes)
    steps = 6
    p0 = torch.from_numpy((rng.standard_normal(total) * 0.02).astype(np.float32)).to(dtype)
    grads = torch.from_numpy((rng.standard_normal((steps, total)) * 1e-3).astype(np.float32)).to(dtype)
    payload = rng.integers(0, 2, total, dtype=np.uint8)
    group = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)

    def run():
        params, off = [], 0
        for n in sizes:
            params.append(torch.nn.Parameter(p0[off:off + n].clone()))
            off += n
        opt = tf.DFCAdamW(params, **group, enable_fiber=True)
        tf.TorchSignFiberChannel(opt).write_bits(0, payload)
        for s in range(steps):
            off = 0
            for p, n in zip(params, sizes):
                p.grad = grads[s, off:off + n].clone()
                off += n
            opt.step()
        p = torch.cat([q.detach().reshape(-1) for q in params]).view(torch.int16).numpy().view(np.uint16)
        m = np.concatenate([opt.state[q]["exp_avg"].reshape(-1).numpy() for q in params]).view(np.uint32)
        v = np.concatenate([opt.state[q]["exp_avg_sq"].reshape(-1).view(torch.int32).numpy()
                            for q in params]).view(np.uint32)
        return p.copy(), m.copy(), v.copy()

    p, m, v = run()
    torch.Tensor.sqrt = _ieee_sqrt
    try:
        pi, m2, v2 = run()
    finally:
        torch.Tensor.sqrt = _stock_sqrt
    assert np.array_equal(m, m2) and np.array_equal(v, v2)
    save(name, sizes=np.array(sizes, np.int64),
         p0=p0.view(torch.int16).numpy().view(np.uint16), grads=grads.view(torch.int16).numpy().view(np.uint16),
         none_mask=np.zeros((steps, len(sizes)), bool), fiber=np.bool_(True), payload=payload,
         p=p, p_ieee_sqrt=pi, m=m, v=v, steps=np.full(len(sizes), steps, np.int64),
         dtype=np.array("bf16" if dtype == torch.bfloat16 else "f16"), **group_arrays(group))


def case_unit_linear(tf):
    torch.manual_seed(17)
    reference = torch.nn.Linear(257, 31)
    lifted = torch.nn.Linear(257, 31)
    lifted.load_state_dict(reference.state_dict())
    w0 = reference.weight.detach().numpy().copy()
    b0 = reference.bias.detach().numpy().copy()
    opt_ref = tf.DFCAdamW(reference.parameters(), lr=3e-4, weight_decay=0.01, enable_fiber=False)
    opt_dfc = tf.DFCAdamW(lifted.parameters(), lr=3e-4, weight_decay=0.01, enable_fiber=True)
    channel = tf.TorchSignFiberChannel(opt_dfc)
    payload = np.random.default_rng(19).bytes(channel.byte_capacity)
    channel.write_bytes(0, payload)
    xs, ys = [], []
    for _ in range(50):
        x = torch.randn(23, 257)
        y = torch.randn(23, 31)
        xs.append(x.numpy().copy())
        ys.append(y.numpy().copy())
        for model, optimizer in ((reference, opt_ref), (lifted, opt_dfc)):
            optimizer.zero_grad()
            torch.nn.functional.mse_loss(model(x), y).backward()
            optimizer.step()
    assert all(torch.equal(a, b) for a, b in zip(reference.parameters(), lifted.parameters()))
    assert channel.read_bytes(0, len(payload)) == payload
    save("unit_linear", w0=w0, b0=b0, x=np.stack(xs), y=np.stack(ys),
         payload=np.frombuffer(payload, np.uint8),
         w=reference.weight.detach().numpy(), b=reference.bias.detach().numpy())


def replay_images(n=24, seed=5):
    rng = np.random.default_rng(seed)
    x = (rng.integers(0, 256, (n, 3, 32, 32)) / 255.0).astype(np.float32)
    flat = x.reshape(n, -1)
    # exact ties k + 0.5 after the FP32 multiply by 15, both parities
    ties = np.array([(k + 0.5) / 15.0 for k in range(15)], np.float32)
    flat[1, :15] = ties
    flat[2, :64] = rng.uniform(-0.5, 1.5, 64).astype(np.float32)
    flat[3, :6] = np.array([-0.0, np.inf, -np.inf, np.nan, 1.0, 0.0], np.float32)
    flat[4] = np.float32(1.0)
    flat[5] = np.float32(0.0)
    labels = rng.integers(0, 100, n)
    tasks = labels // 10
    labels[6], tasks[6] = 65535, 65535
    return x, labels, tasks


def case_replay(vb):
    x, labels, tasks = replay_images()
    codec = vb.CIFAR4BitCodec
    records = np.stack([np.frombuffer(codec.encode(torch.from_numpy(x[i]), int(labels[i]),
                                                   int(tasks[i])), np.uint8)
                        for i in range(len(x))])
    dec = [codec.decode(r.tobytes()) for r in records]
    decoded = np.stack([d[0].numpy().reshape(-1) for d in dec])
    # corruptions: a flipped pixel bit, a flipped CRC bit, a bad magic, a
    # flipped header bit; the error text each raises
    bad = records[:4].copy()
    bad[0, 100] ^= 0x10
    bad[1, 1545] ^= 0x01
    bad[2, 0] = ord("X")
    bad[3, 5] ^= 0x80
    errors = []
    for r in bad:
        try:
            codec.decode(r.tobytes())
            errors.append("")
        except RuntimeError as e:
            errors.append(str(e))
    # reservoir: ArrayChannel with room for 5 records and 100 spare bytes
    channel = vb.ArrayChannel(vb.FiberReservoir.HEADER_BYTES + 5 * codec.RECORD_BYTES + 100)
    res = vb.FiberReservoir(channel)
    rng = np.random.default_rng(11)
    for i in range(12):
        res.add(torch.from_numpy(x[i]), int(labels[i]), int(tasks[i]), rng)
    channel_after_adds = np.frombuffer(bytes(channel.storage), np.uint8).copy()
    sx, sy = res.sample(6, rng)
    save("replay", images=x, labels=labels, tasks=tasks, records=records, decoded=decoded,
         dec_labels=np.array([d[1] for d in dec]), dec_tasks=np.array([d[2] for d in dec]),
         bad_records=bad, bad_errors=np.array(errors), res_capacity=res.capacity,
         res_size=res.size, res_seen=res.seen, res_rng_seed=11, res_adds=12,
         channel=channel_after_adds, sample_x=sx.numpy(), sample_y=sy.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("T3ST_REFERENCE"),
                    required="T3ST_REFERENCE" not in os.environ,
                    help="checkout of the reference (YellowJune/T3st); default: $T3ST_REFERENCE")
    ap.add_argument("--only", default=None, help="make one case (by file name)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "remote"))
    sys.path.insert(0, REPO)
    import torch_fiber as tf  # the reference module
    from oracle import oracle

    torch.set_num_threads(1)
    if args.only == "replay":
        import vision_benchmark as vb  # the reference's benchmark module

        case_replay(vb)
        return
    case_mt(tf, True, "fiber_mt")
    case_mt(tf, False, "plain_mt")
    case_ragged(tf, oracle)
    case_c1(tf)
    case_lowp(tf, torch.bfloat16, "bf16_params")
    case_lowp(tf, torch.float16, "f16_params")
    case_unit_linear(tf)
    import vision_benchmark as vb

    case_replay(vb)


if __name__ == "__main__":
    main()
