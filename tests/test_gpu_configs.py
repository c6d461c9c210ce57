"""The step at full workload sizes, checked bit for bit against the oracle
on sampled tensors plus size-independent properties over everything:

  resnet18    62 FP32 tensors, 11,173,962 params, packed moments warmed for
              10 steps, then one step compared in full with the oracle
  ragged      4096 tensors, ~1.1e9 elements, sizes log-uniform in [1, 4M]
              (forced sizes not multiple of 4 or 8), Student-t(3)*1e-3
              gradients with 5% zeros and 0.1% denormals, moments pre-seeded
              (packed: random 16-bit residual fields; both formats: random
              payload bits), weight decay on; two steps in which ~5% of the
              tensors have no gradient each, so per-tensor step counters
              diverge (0, 1 or 2) and one launch carries several hyper sets;
              every element of every tensor compared with the oracle, in the
              reference's sign-fiber format and in the packed format
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


@pytest.mark.parametrize("fmt", ["fp32", "packed"])
def test_ragged_4096_tensors_every_element(cuda, fmt):
    from concurrent.futures import ThreadPoolExecutor

    sizes = ragged_sizes(0)
    assert len(sizes) == 4096 and sum(sizes) > 1_000_000_000
    mode = O.MODE_PACKED if fmt == "packed" else O.MODE_SIGNFIBER
    lr, betas, eps, wd = 3e-4, (0.8, 0.95), 1e-6, 0.01
    gen = torch.Generator(device=cuda).manual_seed(5)
    params = [torch.nn.Parameter(torch.empty(n, device=cuda).normal_(0, 0.02, generator=gen))
              for n in sizes]
    opt = DFCAdamW(params, lr=lr, betas=betas, eps=eps, weight_decay=wd, moment_format=fmt)
    for p in params:
        st = opt.state[p]
        st["exp_avg"].normal_(0, 1e-3, generator=gen)
        st["exp_avg_sq"].normal_(0, 1e-6, generator=gen).abs_()
        if fmt == "packed":
            for key in ("exp_avg", "exp_avg_sq"):
                st[key].view(torch.int32).copy_(st[key].view(torch.int32) & -65536)
                random_residual_fields_(st[key], gen)
        random_payload_(st["exp_avg_sq"], gen)
    rng = np.random.default_rng(11)
    # step s: the tensors without a gradient (different ones each step)
    skip = [set(rng.choice(len(sizes), 205, replace=False).tolist()) for _ in range(2)]
    # device snapshots of the starting state and of each step's gradients
    snap = [(p.detach().clone(), opt.state[p]["exp_avg"].clone(),
             opt.state[p]["exp_avg_sq"].clone()) for p in params]
    grads = [[None if i in skip[s] else student_t_grads_(torch.empty(n, device=cuda), gen)
              for i, n in enumerate(sizes)] for s in range(2)]
    for s in range(2):
        for p, g in zip(params, grads[s]):
            p.grad = g
        opt.step()
    torch.cuda.synchronize()

    def check(i):
        pp = _host(snap[i][0]).copy()
        m = _host(snap[i][1]).view(np.uint32).copy()
        v = _host(snap[i][2]).view(np.uint32).copy()
        step = 0
        for s in range(2):
            if grads[s][i] is None:
                continue
            step += 1
            O.step(mode, O.reference_hyper(lr, betas, eps, wd, step), pp, _host(grads[s][i]), m, v)
        p = params[i]
        ok = (np.array_equal(_host(p).view(np.uint32), pp.view(np.uint32))
              and np.array_equal(_host(opt.state[p]["exp_avg"]).view(np.uint32), m)
              and np.array_equal(_host(opt.state[p]["exp_avg_sq"]).view(np.uint32), v)
              and opt.state[p]["step"] == step)
        return i, ok, step

    with ThreadPoolExecutor(max_workers=16) as pool:
        results = list(pool.map(check, range(len(sizes))))
    bad = [i for i, ok, _ in results if not ok]
    assert not bad, f"{len(bad)} tensors differ from the oracle, first {bad[:8]}"
    counts = np.bincount([st for _, _, st in results], minlength=3)
    assert counts[0] > 0 and counts[1] > 300 and counts[2] > 3000, counts


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
