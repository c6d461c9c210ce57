"""The step at full workload sizes, checked bit for bit against the oracle
on sampled tensors plus size-independent properties over everything:

  resnet18    62 FP32 tensors, 11,173,962 params, packed moments warmed for
              10 steps, then one step compared in full with the oracle
  ragged      4096 tensors, ~1.1e9 elements, sizes log-uniform in [1, 4M]
              (forced sizes not multiple of 4 or 8), Student-t(3)*1e-3
              gradients with 5% zeros and 0.1% denormals, packed moments with
              random 16-bit residual fields and random payload bits; one
              step; 64 tensors compared with the oracle, every payload bit of
              every tensor checked
  flat 2^30   ZeRO-1 path on one GPU with bf16 error-feedback compression;
              sampled slices compared with the oracle (compression + step)
"""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from t3st_b200 import DFCAdamW
from t3st_b200.workloads import (random_payload_, random_residual_fields_, ragged_sizes,
                                 resnet18_cifar_shapes, student_t_grads_)

pytestmark = pytest.mark.gpu


def _host(t):
    return t.detach().reshape(-1).cpu().numpy()


def test_resnet18_multitensor_step_full_size(cuda):
    gen = torch.Generator(device=cuda).manual_seed(0)
    params = [torch.nn.Parameter(torch.empty(s, device=cuda).normal_(0, 0.02, generator=gen))
              for s in resnet18_cifar_shapes()]
    assert sum(p.numel() for p in params) == 11_173_962
    opt = DFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed")
    for _ in range(10):
        for p in params:
            p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
        opt.step()
    for p in params:
        p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
    before = [(_host(p).copy(), _host(p.grad).copy(),
               _host(opt.state[p]["exp_avg"]).view(np.uint32).copy(),
               _host(opt.state[p]["exp_avg_sq"]).view(np.uint32).copy()) for p in params]
    opt.step()
    torch.cuda.synchronize()
    h = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 11)
    for p, (pp, g, m, v) in zip(params, before):
        O.step(O.MODE_PACKED, h, pp, g, m, v)
        np.testing.assert_array_equal(_host(p).view(np.uint32), pp.view(np.uint32))
        np.testing.assert_array_equal(_host(opt.state[p]["exp_avg"]).view(np.uint32), m)
        np.testing.assert_array_equal(_host(opt.state[p]["exp_avg_sq"]).view(np.uint32), v)


def test_ragged_4096_tensors_full_size(cuda):
    sizes = ragged_sizes(0)
    assert len(sizes) == 4096 and sum(sizes) > 1_000_000_000
    gen = torch.Generator(device=cuda).manual_seed(5)
    params, grads = [], []
    for n in sizes:
        params.append(torch.nn.Parameter(torch.empty(n, device=cuda).normal_(0, 0.02, generator=gen)))
        grads.append(student_t_grads_(torch.empty(n, device=cuda), gen))
    opt = DFCAdamW(params, lr=3e-4, betas=(0.8, 0.95), eps=1e-6, moment_format="packed")
    for p, g in zip(params, grads):
        st = opt.state[p]
        st["exp_avg"].normal_(0, 1e-3, generator=gen)
        st["exp_avg_sq"].normal_(0, 1e-6, generator=gen).abs_()
        for key in ("exp_avg", "exp_avg_sq"):
            st[key].view(torch.int32).copy_(st[key].view(torch.int32) & -65536)
            random_residual_fields_(st[key], gen)
        random_payload_(st["exp_avg_sq"], gen)
        p.grad = g
    rng = np.random.default_rng(1)
    sample = sorted(set(range(26)) | set(rng.choice(len(sizes), 38, replace=False).tolist()))
    before = {i: (_host(params[i]).copy(), _host(grads[i]).copy(),
                  _host(opt.state[params[i]]["exp_avg"]).view(np.uint32).copy(),
                  _host(opt.state[params[i]]["exp_avg_sq"]).view(np.uint32).copy()) for i in sample}
    payload = [(opt.state[p]["exp_avg_sq"].view(torch.int32) < 0) for p in params]
    opt.step()
    torch.cuda.synchronize()
    h = O.reference_hyper(3e-4, (0.8, 0.95), 1e-6, 0.0, 1)
    for i in sample:
        pp, g, m, v = before[i]
        O.step(O.MODE_PACKED, h, pp, g, m, v)
        p = params[i]
        np.testing.assert_array_equal(_host(p).view(np.uint32), pp.view(np.uint32), err_msg=str(i))
        np.testing.assert_array_equal(_host(opt.state[p]["exp_avg"]).view(np.uint32), m)
        np.testing.assert_array_equal(_host(opt.state[p]["exp_avg_sq"]).view(np.uint32), v)
    bad = sum(int(torch.count_nonzero((opt.state[p]["exp_avg_sq"].view(torch.int32) < 0) != b))
              for p, b in zip(params, payload))
    assert bad == 0
    assert all(opt.state[p]["step"] == 1 for p in params)


def test_zero1_flat_2pow30_one_gpu(cuda):
    from t3st_b200.zero import ShardedDFCAdamW

    P = 1 << 30
    gen = torch.Generator(device=cuda).manual_seed(9)
    param = torch.nn.Parameter(torch.empty(P, device=cuda).normal_(0, 0.02, generator=gen))
    opt = ShardedDFCAdamW([param], lr=1e-3, weight_decay=0.01, compress_grads=True)
    del param
    opt.flat_grad[:P].normal_(0, 1e-3, generator=gen)
    starts = [0, 12345, (1 << 28) + 7, P - 70000]
    n = 65536
    snap = [(_host(opt.flat_param[s:s + n]).copy(), _host(opt.flat_grad[s:s + n]).copy())
            for s in starts]
    opt.step()
    torch.cuda.synchronize()
    h = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 1)
    for s, (pp, g) in zip(starts, snap):
        c = np.zeros(n, np.uint16)
        q = np.zeros(n, np.uint16)
        O.compress_ef(g, c, q)
        np.testing.assert_array_equal(_host(opt.comp[s:s + n]).view(np.uint16), c)
        np.testing.assert_array_equal(_host(opt.resid[s:s + n]).view(np.uint16), q)
        m = np.zeros(n, np.uint32)
        v = np.zeros(n, np.uint32)
        O.step(O.MODE_PACKED, h, pp, c, m, v)
        np.testing.assert_array_equal(_host(opt.flat_param[s:s + n]).view(np.uint32), pp.view(np.uint32))
        np.testing.assert_array_equal(_host(opt.exp_avg[s:s + n]).view(np.uint32), m)
