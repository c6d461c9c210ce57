"""Native steady-state plan of DFCAdamW.step() (t3st_b200._dfc_host), on CPU.

The plan is built over CPU tensors, and its launch function is a recorder
with dfc_mt_step's signature, so no kernel runs.  The tests check that the
plan:
- forms the hyper sets bit for bit like the Python hyper_row
  (remote/torch_fiber.py:75-116);
- follows gradients that PyTorch re-creates every step, advances every
  state["step"], and hands the launcher the current pointers;
- refuses, with no side effect, what it cannot follow: a missing gradient, a
  storage swapped under the same tensor, other strides, unequal step
  counters, a rebound param_groups or state, a tensor learning rate, a
  parameter added to a group;
- passes a launch error through as the status and leaves the counters alone.
"""

import ctypes
import gc
import weakref

import numpy as np
import pytest
import torch

from t3st_b200 import DFCAdamW, _lib
from t3st_b200 import torch_fiber as tf

LAUNCH = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                          ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p)


class Recorder:
    def __init__(self, status=0):
        self.calls = []
        self.status = status
        self.fn = LAUNCH(self._call)
        self.address = ctypes.cast(self.fn, ctypes.c_void_p).value

    def _call(self, segs, n, hyp, nh, mode, scale, stream):
        raw = (ctypes.c_uint8 * (n * _lib.SEGMENT_DTYPE.itemsize)).from_address(segs)
        rawh = (ctypes.c_uint8 * (nh * _lib.HYPER_DTYPE.itemsize)).from_address(hyp)
        self.calls.append((np.frombuffer(raw, dtype=_lib.SEGMENT_DTYPE).copy(),
                           np.frombuffer(rawh, dtype=_lib.HYPER_DTYPE).copy(), mode, scale, stream))
        return self.status


def _setup(shapes=((3, 5), (7,), (2, 2, 2)), groups=1, status=0, **kw):
    params = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    for p in params:
        p.grad = torch.zeros_like(p)
    if groups == 1:
        opt = DFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed", **kw)
    else:
        opt = DFCAdamW([{"params": params[:1]}, {"params": params[1:], "lr": 3e-4,
                                                 "weight_decay": 0.0}],
                       lr=1e-3, weight_decay=0.01, moment_format="packed", **kw)
    work = [(p, opt.state[p], p.grad, gi) for gi, g in enumerate(opt.param_groups)
            for p in g["params"]]
    segs = np.zeros(len(work), dtype=_lib.SEGMENT_DTYPE)
    segs["param"] = [p.data_ptr() for p in params]
    segs["grad"] = [p.grad.data_ptr() for p in params]
    segs["numel"] = [p.numel() for p in params]
    rec = Recorder(status)
    plan = tf._native_plan(opt, work, segs, torch.device("cuda", 0), launch=rec.address)
    assert plan is not None
    return params, opt, plan, rec


@pytest.mark.parametrize("lr,b1,b2,eps,wd", [
    (1e-3, 0.9, 0.999, 1e-8, 0.01), (3e-4, 0.8, 0.95, 1e-6, 0.0), (1, 0.0, 0.5, 1e-12, 1e-4),
    (0.1, 0.99, 0.9999, 0, -0.0), (2.5e-5, 0.5, 0.999999, 1e-30, 5)])
def test_native_hyper_rows_match_python(lr, b1, b2, eps, wd):
    host = _lib.host()
    for step in (1, 2, 3, 10, 100, 1000, 12345, 10 ** 6, 2 ** 31 + 5):
        want = np.array([tf.hyper_row(lr, (b1, b2), eps, wd, step)], dtype=_lib.HYPER_DTYPE)[0]
        got = host.hyper_row(lr, b1, b2, eps, wd, step)
        want_bits = np.array([want[f] for f in _lib.HYPER_FIELDS], dtype=np.float32).view(np.uint32)
        got_bits = np.array(got, dtype=np.float32).view(np.uint32)
        np.testing.assert_array_equal(got_bits, want_bits, err_msg=f"step {step}")


def test_native_plan_follows_new_gradient_tensors():
    params, opt, plan, rec = _setup()
    for step in range(1, 4):
        for p in params:  # what backward does after zero_grad(set_to_none=True)
            p.grad = torch.full_like(p, float(step))
        assert plan.step(0) == 1
        segs, hyp, mode, scale, stream = rec.calls[-1]
        np.testing.assert_array_equal(segs["grad"], [p.grad.data_ptr() for p in params])
        np.testing.assert_array_equal(segs["param"], [p.data_ptr() for p in params])
        assert mode == _lib.MODE_PACKED and not scale and not stream
        want = np.array([tf.hyper_row(1e-3, (0.9, 0.999), 1e-8, 0.01, step)],
                        dtype=_lib.HYPER_DTYPE)
        assert hyp.tobytes() == want.tobytes()
        assert all(opt.state[p]["step"] == step for p in params)


def test_native_plan_one_hyper_set_per_group():
    params, opt, plan, rec = _setup(groups=2)
    assert plan.step(0) == 1
    segs, hyp, *_ = rec.calls[-1]
    assert list(segs["hyper"]) == [0, 1, 1]
    want = np.array([tf.hyper_row(1e-3, (0.9, 0.999), 1e-8, 0.01, 1),
                     tf.hyper_row(3e-4, (0.9, 0.999), 1e-8, 0.0, 1)], dtype=_lib.HYPER_DTYPE)
    assert hyp.tobytes() == want.tobytes()
    opt.param_groups[1]["lr"] = 1e-2  # a scheduler's change is read every step
    assert plan.step(0) == 1
    want = np.array([tf.hyper_row(1e-2, (0.9, 0.999), 1e-8, 0.0, 2)], dtype=_lib.HYPER_DTYPE)
    assert rec.calls[-1][1][1:].tobytes() == want.tobytes()


def _refused(plan, opt, params, rec):
    before = [opt.state[p]["step"] for p in params]
    n = len(rec.calls)
    assert plan.step(0) == 0
    assert len(rec.calls) == n
    assert [opt.state[p]["step"] for p in params] == before


def test_native_plan_refuses_what_it_cannot_follow():
    params, opt, plan, rec = _setup()
    assert plan.step(0) == 1
    g = params[0].grad
    g.set_(torch.zeros_like(g))          # same tensor object, new storage
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    params[1].grad = None                # a parameter without gradient
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    params[2].grad = torch.zeros(params[2].shape[::-1]).permute(2, 1, 0)  # other strides
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    params[2].grad_dtype = None          # allow a gradient of another dtype
    params[2].grad = torch.zeros_like(params[2], dtype=torch.float64)
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    opt.state[params[1]]["step"] = 7      # per-tensor counters that differ
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    opt.param_groups[0]["lr"] = torch.tensor(1e-3)  # a tensor learning rate
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    opt.param_groups[0]["params"].append(torch.nn.Parameter(torch.zeros(2)))
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    opt.param_groups = list(opt.param_groups)  # rebound (load_state_dict does this)
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    opt.enable_fiber = False             # another moment mode
    _refused(plan, opt, params, rec)

    params, opt, plan, rec = _setup()
    params[0].data = torch.zeros_like(params[0])  # the parameter's storage moved
    _refused(plan, opt, params, rec)


def test_native_plan_passes_launch_errors_through():
    params, opt, plan, rec = _setup(status=_lib.DFC_ERR_ALIGN)
    assert plan.step(0) == _lib.DFC_ERR_ALIGN
    assert all(opt.state[p]["step"] == 0 for p in params)


def test_native_plan_is_collected_with_its_optimizer():
    params, opt, plan, rec = _setup()
    opt._native = plan                  # the optimizer holds its plan; the plan holds opt.__dict__
    del plan
    ref = weakref.ref(opt)
    del opt
    gc.collect()
    assert ref() is None


def test_step_uses_hook_wrapper_only_when_needed():
    """DFCAdamW.step is not wrapped by torch.optim.Optimizer; registered
    hooks still run, through the same wrapper (profiler range, hooks)."""
    assert getattr(DFCAdamW.step, "hooked", False)
    params, opt, plan, rec = _setup()
    seen = []
    opt.register_step_pre_hook(lambda o, a, k: seen.append("pre"))
    opt.register_step_post_hook(lambda o, a, k: seen.append("post"))
    # the general path runs on CUDA tensors only, so the wrapped step raises
    # here -- after the pre-hook ran
    with pytest.raises(RuntimeError, match="CUDA"):
        opt.step()
    assert seen == ["pre"]
