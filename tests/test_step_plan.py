"""Host logic of DFCAdamW's steady-state step plan, on CPU with the library
call replaced by a recorder (no kernel runs).

After a first step the optimizer keeps its segment descriptors.  Each later
step only re-reads pointers, dtypes and step counters.  These tests check
that the plan follows gradients that PyTorch re-creates every step
(zero_grad(set_to_none=True), then backward) without a rebuild.  They also
check that it refuses a storage swapped under the same tensor, a dtype
change and a missing gradient, so the general path re-validates those."""

import types

import numpy as np
import torch

from t3st_b200 import DFCAdamW, _lib
from t3st_b200 import torch_fiber as tf


def _setup(monkeypatch, shapes=((3, 5), (7,), (2, 2, 2))):
    params = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    for p in params:
        p.grad = torch.zeros_like(p)
    opt = DFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed")
    work = [(p, opt.state[p], p.grad, 0) for p in params]
    segs = np.zeros(len(work), dtype=_lib.SEGMENT_DTYPE)
    segs["param"] = [p.data_ptr() for p in params]
    segs["grad"] = [p.grad.data_ptr() for p in params]
    opt._fast = tf._FastPlan(opt, work, segs, torch.device("cuda", 0))
    calls = []

    def mt_step(segs_ptr, n, hyp_ptr, n_hyp, mode, scale, stream):
        arr = np.ctypeslib.as_array(
            (np.ctypeslib.ctypes.c_uint8 * (n * _lib.SEGMENT_DTYPE.itemsize)).from_address(segs_ptr))
        calls.append(arr.view(_lib.SEGMENT_DTYPE).copy())
        return 0

    monkeypatch.setattr(_lib, "lib", lambda: types.SimpleNamespace(dfc_mt_step=mt_step))
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "current_stream",
                        lambda dev=None: types.SimpleNamespace(cuda_stream=0))
    return params, opt, calls


def test_plan_follows_new_gradient_tensors(monkeypatch):
    params, opt, calls = _setup(monkeypatch)
    fast = opt._fast
    for step in range(1, 4):
        for p in params:  # what backward does after zero_grad(set_to_none=True)
            p.grad = torch.full_like(p, float(step))
        assert fast.try_step(opt)
        np.testing.assert_array_equal(calls[-1]["grad"], [p.grad.data_ptr() for p in params])
        np.testing.assert_array_equal(calls[-1]["param"], [p.data_ptr() for p in params])
        assert all(opt.state[p]["step"] == step for p in params)


def test_plan_refuses_what_it_cannot_follow(monkeypatch):
    params, opt, calls = _setup(monkeypatch)
    fast = opt._fast
    assert fast.try_step(opt)
    g = params[0].grad
    g.set_(torch.zeros_like(g))          # same tensor object, new storage
    assert not fast.try_step(opt)
    params, opt, calls = _setup(monkeypatch)
    params[1].grad = None                # a parameter without gradient
    assert not opt._fast.try_step(opt)
    params, opt, calls = _setup(monkeypatch)
    params[2].grad = torch.zeros(params[2].shape[::-1]).permute(2, 1, 0)  # other strides
    assert not opt._fast.try_step(opt)
    assert not calls


def test_copy_and_pickle_keep_format_and_drop_plans():
    """An optimizer that is deep-copied or pickled keeps its moment format
    and options, and rebuilds its step plans on the next step."""
    import copy
    import pickle

    params = [torch.nn.Parameter(torch.zeros(3))]
    opt = DFCAdamW(params, lr=1e-3, enable_fiber=False, moment_format="packed",
                   max_grad_norm=2.0)
    opt._native = object()  # stands for a plan bound to the original's storage
    for twin in (copy.deepcopy(opt), pickle.loads(pickle.dumps(opt))):
        assert twin.enable_fiber is False and twin.moment_format == "packed"
        assert twin.max_grad_norm == 2.0
        assert twin._native is None and twin._fast is None and twin._plan_key is None
        assert twin.mode == _lib.MODE_PACKED
        assert twin.param_groups[0]["lr"] == 1e-3


def test_load_state_dict_keeps_format_and_options():
    """torch.optim.Optimizer.load_state_dict re-enters __setstate__ with state
    and param_groups only; the optimizer's own format and options stay."""
    params = [torch.nn.Parameter(torch.zeros(3))]
    opt = DFCAdamW(params, lr=1e-3, enable_fiber=False, moment_format="packed",
                   max_grad_norm=2.0)
    opt.load_state_dict(opt.state_dict())  # same format: no conversion needed
    assert opt.moment_format == "packed" and opt.enable_fiber is False
    assert opt.max_grad_norm == 2.0 and opt.mode == _lib.MODE_PACKED
