// Steady-state host path of DFCAdamW.step() (remote/torch_fiber.py:68-117),
// as a CPython extension: t3st_b200._dfc_host.StepPlan.
//
// After a step through the general (validating) Python path, the optimizer
// keeps one StepPlan.  Every later step() re-checks, at C speed, exactly the
// conditions under which the segment descriptors of that step still hold:
//   - the parameter groups hold the same parameter objects, in order, and
//     their lr / betas / eps / weight_decay are plain Python numbers;
//   - every parameter still has its storage (same data pointer) and a
//     gradient; a gradient tensor that PyTorch re-created since the last step
//     (zero_grad(set_to_none=True), then backward) is followed when its
//     dtype, sizes and strides match: only its pointer changes;
//   - every state["step"] is the same Python int.
// It then forms the per-group hyper sets exactly like hyper_row() in
// torch_fiber.py (double arithmetic, one rounding to FP32), calls dfc_mt_step
// of libdfc_b200.so (through a function pointer handed over by the Python
// side) on the caller's current CUDA stream, and advances every
// state["step"].  Any mismatch returns 0 without side effects, and the Python
// side re-validates everything through its general path.
//
// The plan holds no device memory and launches nothing itself; the C ABI is
// still the only way into the kernels.

#include <Python.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>

#include <cmath>
#include <cstdint>
#include <vector>

#include "dfc_b200.h"

namespace {

using LaunchFn = int (*)(const DfcSegment*, int32_t, const DfcHyper*, int32_t, int32_t,
                         const float*, void*);

PyObject* k_params = nullptr;
PyObject* k_param_groups = nullptr;
PyObject* k_step = nullptr;
PyObject* k_lr = nullptr;
PyObject* k_betas = nullptr;
PyObject* k_eps = nullptr;
PyObject* k_wd = nullptr;

struct GradInfo {
  at::Tensor tensor;              // the gradient seen by the last step (identity check)
  c10::ScalarType dtype;
  std::vector<int64_t> sizes, strides;
};

struct Plan {
  PyObject_HEAD
  int32_t n;          // segments (= parameters, in param_groups order)
  int32_t n_groups;
  int32_t mode;
  int32_t device;     // CUDA device index of every parameter
  LaunchFn launch;
  DfcSegment* segs;   // inside segs_owner's buffer
  DfcHyper* hyp;      // inside hyp_owner's buffer
  PyObject* segs_owner;
  PyObject* hyp_owner;
  PyObject* groups;   // the optimizer's param_groups list
  PyObject* owner;    // the optimizer's instance __dict__
  PyObject* watch;    // tuple of (key, object) pairs: owner[key] must still be object
  std::vector<PyObject*>* params;   // strong references
  std::vector<PyObject*>* states;   // strong references
  std::vector<Py_ssize_t>* group_len;
  std::vector<GradInfo>* grads;
};

// A plain Python number as a double (ints and floats only: anything else,
// e.g. a tensor learning rate, sends the step to the general path).
bool number(PyObject* o, double* out) {
  if (PyFloat_CheckExact(o)) {
    *out = PyFloat_AS_DOUBLE(o);
    return true;
  }
  if (PyLong_CheckExact(o)) {
    *out = PyLong_AsDouble(o);
    if (*out == -1.0 && PyErr_Occurred()) {
      PyErr_Clear();
      return false;
    }
    return true;
  }
  return false;
}

// hyper_row() of torch_fiber.py for one group at step s: every value formed
// in double as Python forms it (float ** int is C pow, math.sqrt is C sqrt),
// then rounded once to FP32.
bool group_hyper(PyObject* group, long long s, DfcHyper* h) {
  if (!PyDict_Check(group)) return false;
  PyObject* lr_o = PyDict_GetItem(group, k_lr);
  PyObject* betas = PyDict_GetItem(group, k_betas);
  PyObject* eps_o = PyDict_GetItem(group, k_eps);
  PyObject* wd_o = PyDict_GetItem(group, k_wd);
  if (!lr_o || !betas || !eps_o || !wd_o) return false;
  if (!(PyTuple_CheckExact(betas) || PyList_CheckExact(betas)) || PySequence_Fast_GET_SIZE(betas) < 2)
    return false;
  double lr, b1, b2, eps, wd;
  if (!number(lr_o, &lr) || !number(eps_o, &eps) || !number(wd_o, &wd) ||
      !number(PySequence_Fast_GET_ITEM(betas, 0), &b1) ||
      !number(PySequence_Fast_GET_ITEM(betas, 1), &b2))
    return false;
  const double sd = static_cast<double>(s);
  const double bc1 = 1.0 - std::pow(b1, sd);
  const double bc2 = 1.0 - std::pow(b2, sd);
  const double decay = wd != 0.0 ? 1.0 - lr * wd : 1.0;
  h->beta1 = static_cast<float>(b1);
  h->one_minus_beta1 = static_cast<float>(1.0 - b1);
  h->beta2 = static_cast<float>(b2);
  h->one_minus_beta2 = static_cast<float>(1.0 - b2);
  h->sqrt_bc2 = static_cast<float>(std::sqrt(bc2));
  h->eps = static_cast<float>(eps);
  h->decay = static_cast<float>(decay);
  h->neg_step_size = static_cast<float>(-(lr / bc1));
  h->grad_scale = 1.0f;
  h->reserved[0] = h->reserved[1] = h->reserved[2] = 0.0f;
  return true;
}

bool same_layout(const at::Tensor& g, const GradInfo& gi) {
  return g.layout() == c10::kStrided && g.scalar_type() == gi.dtype &&
         g.sizes().equals(gi.sizes) && g.strides().equals(gi.strides);
}

// Returns 1 (launched), 0 (the plan does not hold: use the general path) or
// the negative status of dfc_mt_step.
int run_step(Plan* self, bool explicit_stream, void* stream) {
  const int32_t n = self->n;
  std::vector<PyObject*>& params = *self->params;
  if (!self->owner || !self->groups) return 0;
  // 0. the optimizer attributes the plan depends on are the same objects
  for (Py_ssize_t w = 0; w < PyTuple_GET_SIZE(self->watch); ++w) {
    PyObject* kv = PyTuple_GET_ITEM(self->watch, w);
    if (PyDict_GetItem(self->owner, PyTuple_GET_ITEM(kv, 0)) != PyTuple_GET_ITEM(kv, 1)) return 0;
  }
  // 1. the parameter groups hold the plan's parameters, in order
  if (!PyList_CheckExact(self->groups) || PyList_GET_SIZE(self->groups) != self->n_groups) return 0;
  {
    Py_ssize_t k = 0;
    for (int32_t gi = 0; gi < self->n_groups; ++gi) {
      PyObject* group = PyList_GET_ITEM(self->groups, gi);
      if (!PyDict_Check(group)) return 0;
      PyObject* plist = PyDict_GetItem(group, k_params);
      if (!plist || !PyList_CheckExact(plist) ||
          PyList_GET_SIZE(plist) != (*self->group_len)[gi])
        return 0;
      for (Py_ssize_t j = 0; j < PyList_GET_SIZE(plist); ++j)
        if (PyList_GET_ITEM(plist, j) != params[k++]) return 0;
    }
  }
  // 2. one shared step counter (per-tensor counters, :85-86)
  long long s = 0;
  for (int32_t i = 0; i < n; ++i) {
    PyObject* sv = PyDict_GetItem((*self->states)[i], k_step);
    if (!sv || !PyLong_CheckExact(sv)) return 0;
    const long long v = PyLong_AsLongLong(sv);
    if (v == -1 && PyErr_Occurred()) {
      PyErr_Clear();
      return 0;
    }
    if (i == 0) s = v;
    else if (v != s) return 0;
  }
  if (s < 0 || s >= (1LL << 53) - 1) return 0;
  ++s;
  // 3. hyper sets, into a local copy until every check has passed
  DfcHyper hyp[64];
  if (self->n_groups > 64) return 0;
  for (int32_t gi = 0; gi < self->n_groups; ++gi)
    if (!group_hyper(PyList_GET_ITEM(self->groups, gi), s, &hyp[gi])) return 0;
  // 4. parameter storage unchanged; gradients present (new ones followed)
  std::vector<GradInfo>& grads = *self->grads;
  std::vector<std::pair<int32_t, const at::Tensor*>> renewed;
  for (int32_t i = 0; i < n; ++i) {
    const at::Tensor& p = THPVariable_Unpack(params[i]);
    if (!p.has_storage() || p.data_ptr() != self->segs[i].param) return 0;
    const at::Tensor& g = p.unsafeGetTensorImpl()->grad();
    if (!g.defined()) return 0;
    if (g.unsafeGetTensorImpl() == grads[i].tensor.unsafeGetTensorImpl()) {
      if (!g.has_storage() || g.data_ptr() != self->segs[i].grad) return 0;  // storage swapped
    } else {
      if (!same_layout(g, grads[i]) || g.device() != p.device() || !g.has_storage()) return 0;
      renewed.emplace_back(i, &g);
    }
  }
  // 5. commit: pointers of re-created gradients, hyper sets, launch, counters
  for (auto& r : renewed) {
    self->segs[r.first].grad = r.second->data_ptr();
    grads[r.first].tensor = *r.second;
  }
  for (int32_t gi = 0; gi < self->n_groups; ++gi) self->hyp[gi] = hyp[gi];
  int rc;
  if (explicit_stream) {
    rc = self->launch(self->segs, n, self->hyp, self->n_groups, self->mode, nullptr, stream);
  } else {
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(self->device));
    void* st = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(self->device)).stream();
    rc = self->launch(self->segs, n, self->hyp, self->n_groups, self->mode, nullptr, st);
  }
  if (rc != DFC_OK) return rc < 0 ? rc : -rc;
  PyObject* sobj = PyLong_FromLongLong(s);
  if (!sobj) return -1000;
  for (int32_t i = 0; i < n; ++i) {
    if (PyDict_SetItem((*self->states)[i], k_step, sobj) != 0) {
      Py_DECREF(sobj);
      return -1000;
    }
  }
  Py_DECREF(sobj);
  return 1;
}

// StepPlan.step(stream=None) -> int
//   stream: a cudaStream_t as an int; default: PyTorch's current stream of
//   the plan's device (with that device made current for the launch).
PyObject* plan_step(PyObject* o, PyObject* const* args, Py_ssize_t nargs) {
  Plan* self = reinterpret_cast<Plan*>(o);
  bool explicit_stream = false;
  void* stream = nullptr;
  if (nargs > 1) {
    PyErr_SetString(PyExc_TypeError, "step() takes at most one argument (stream)");
    return nullptr;
  }
  if (nargs == 1 && args[0] != Py_None) {
    explicit_stream = true;
    stream = PyLong_AsVoidPtr(args[0]);
    if (PyErr_Occurred()) return nullptr;
  }
  int rc;
  try {
    rc = run_step(self, explicit_stream, stream);
  } catch (const std::exception& e) {
    PyErr_SetString(PyExc_RuntimeError, e.what());
    return nullptr;
  }
  if (rc == -1000) return nullptr;  // a Python error is set
  return PyLong_FromLong(rc);
}

int plan_traverse(PyObject* o, visitproc visit, void* arg) {
  Plan* self = reinterpret_cast<Plan*>(o);
  if (self->params)
    for (PyObject* p : *self->params) Py_VISIT(p);
  if (self->states)
    for (PyObject* s : *self->states) Py_VISIT(s);
  Py_VISIT(self->segs_owner);
  Py_VISIT(self->hyp_owner);
  Py_VISIT(self->groups);
  Py_VISIT(self->owner);
  Py_VISIT(self->watch);
  return 0;
}

int plan_clear(PyObject* o) {
  Plan* self = reinterpret_cast<Plan*>(o);
  if (self->params) {
    std::vector<PyObject*> v;
    v.swap(*self->params);
    for (PyObject* p : v) Py_DECREF(p);
  }
  if (self->states) {
    std::vector<PyObject*> v;
    v.swap(*self->states);
    for (PyObject* s : v) Py_DECREF(s);
  }
  Py_CLEAR(self->groups);
  Py_CLEAR(self->owner);
  Py_CLEAR(self->watch);
  // the descriptor buffers stay referenced until deallocation: segs and hyp
  // point into them
  return 0;
}

void plan_dealloc(PyObject* o) {
  Plan* self = reinterpret_cast<Plan*>(o);
  PyObject_GC_UnTrack(o);
  plan_clear(o);
  delete self->params;
  delete self->states;
  delete self->group_len;
  delete self->grads;
  Py_CLEAR(self->segs_owner);
  Py_CLEAR(self->hyp_owner);
  Py_TYPE(o)->tp_free(o);
}

// StepPlan(params, states, groups, segs, hypers, mode, device, launch_fn,
//          owner, watch_keys)
//   params  list of parameters in param_groups order (exact torch.Tensor /
//           nn.Parameter objects), one segment each
//   states  their state dicts, same order
//   groups  the optimizer's param_groups list
//   segs    numpy DfcSegment array (n entries, filled by the Python side:
//           pointers, sizes, types, hyper = group index)
//   hypers  numpy DfcHyper array (one per group), rewritten every step
//   mode    DFC_MODE_*
//   device  CUDA device index of every parameter
//   launch_fn  address of dfc_mt_step
//   owner   the optimizer's __dict__
//   watch_keys  tuple of keys of owner whose values must stay the same
//           objects (param_groups, state, the moment format, ...)
PyObject* plan_new(PyTypeObject* type, PyObject* args, PyObject* kwargs) {
  PyObject *params, *states, *groups, *segs, *hypers, *owner, *keys;
  int mode, device;
  unsigned long long launch;
  if (!PyArg_ParseTuple(args, "O!O!O!OOiiKO!O!", &PyList_Type, &params, &PyList_Type, &states,
                        &PyList_Type, &groups, &segs, &hypers, &mode, &device, &launch,
                        &PyDict_Type, &owner, &PyTuple_Type, &keys))
    return nullptr;
  if (PyDict_GetItem(owner, k_param_groups) != groups) {
    PyErr_SetString(PyExc_ValueError, "owner['param_groups'] must be groups");
    return nullptr;
  }
  PyObject* watch = PyTuple_New(PyTuple_GET_SIZE(keys));
  if (!watch) return nullptr;
  for (Py_ssize_t w = 0; w < PyTuple_GET_SIZE(keys); ++w) {
    PyObject* key = PyTuple_GET_ITEM(keys, w);
    PyObject* val = PyDict_GetItem(owner, key);
    PyObject* kv = val ? PyTuple_Pack(2, key, val) : nullptr;
    if (!kv) {
      Py_DECREF(watch);
      if (!PyErr_Occurred()) PyErr_Format(PyExc_KeyError, "owner has no %R", key);
      return nullptr;
    }
    PyTuple_SET_ITEM(watch, w, kv);
  }
  const Py_ssize_t n = PyList_GET_SIZE(params);
  if (PyList_GET_SIZE(states) != n || n == 0 || n > INT32_MAX) {
    Py_DECREF(watch);
    PyErr_SetString(PyExc_ValueError, "params and states must be non-empty lists of one length");
    return nullptr;
  }
  if (PyList_GET_SIZE(groups) == 0 || PyList_GET_SIZE(groups) > 64) {
    Py_DECREF(watch);
    PyErr_SetString(PyExc_ValueError, "1 to 64 parameter groups");
    return nullptr;
  }
  Py_buffer sb, hb;
  if (PyObject_GetBuffer(segs, &sb, PyBUF_WRITABLE | PyBUF_C_CONTIGUOUS) != 0) {
    Py_DECREF(watch);
    return nullptr;
  }
  const bool segs_ok = sb.len == n * static_cast<Py_ssize_t>(sizeof(DfcSegment));
  void* segs_buf = sb.buf;
  PyBuffer_Release(&sb);
  if (!segs_ok) {
    Py_DECREF(watch);
    PyErr_SetString(PyExc_ValueError, "segs must hold one DfcSegment per parameter");
    return nullptr;
  }
  if (PyObject_GetBuffer(hypers, &hb, PyBUF_WRITABLE | PyBUF_C_CONTIGUOUS) != 0) {
    Py_DECREF(watch);
    return nullptr;
  }
  const bool hyp_ok = hb.len == PyList_GET_SIZE(groups) * static_cast<Py_ssize_t>(sizeof(DfcHyper));
  void* hyp_buf = hb.buf;
  PyBuffer_Release(&hb);
  if (!hyp_ok) {
    Py_DECREF(watch);
    PyErr_SetString(PyExc_ValueError, "hypers must hold one DfcHyper per parameter group");
    return nullptr;
  }
  Plan* self = reinterpret_cast<Plan*>(type->tp_alloc(type, 0));
  if (!self) {
    Py_DECREF(watch);
    return nullptr;
  }
  self->n = static_cast<int32_t>(n);
  self->n_groups = static_cast<int32_t>(PyList_GET_SIZE(groups));
  self->mode = mode;
  self->device = device;
  self->launch = reinterpret_cast<LaunchFn>(static_cast<uintptr_t>(launch));
  self->segs = static_cast<DfcSegment*>(segs_buf);
  self->hyp = static_cast<DfcHyper*>(hyp_buf);
  Py_INCREF(segs);
  Py_INCREF(hypers);
  Py_INCREF(groups);
  self->segs_owner = segs;
  self->hyp_owner = hypers;
  self->groups = groups;
  Py_INCREF(owner);
  self->owner = owner;
  self->watch = watch;
  self->params = new std::vector<PyObject*>();
  self->states = new std::vector<PyObject*>();
  self->group_len = new std::vector<Py_ssize_t>();
  self->grads = new std::vector<GradInfo>();
  PyObject* fail = nullptr;
  try {
    for (Py_ssize_t i = 0; i < n; ++i) {
      PyObject* p = PyList_GET_ITEM(params, i);
      PyObject* st = PyList_GET_ITEM(states, i);
      if (!THPVariable_CheckExact(p) || !PyDict_Check(st)) {
        fail = PyExc_TypeError;
        break;
      }
      Py_INCREF(p);
      Py_INCREF(st);
      self->params->push_back(p);
      self->states->push_back(st);
      const at::Tensor& g = THPVariable_Unpack(p).unsafeGetTensorImpl()->grad();
      if (!g.defined() || g.data_ptr() != self->segs[i].grad) {
        fail = PyExc_ValueError;
        break;
      }
      GradInfo gi;
      gi.tensor = g;
      gi.dtype = g.scalar_type();
      gi.sizes = g.sizes().vec();
      gi.strides = g.strides().vec();
      self->grads->push_back(std::move(gi));
    }
  } catch (const std::exception& e) {
    Py_DECREF(self);
    PyErr_SetString(PyExc_RuntimeError, e.what());
    return nullptr;
  }
  if (fail) {
    Py_DECREF(self);
    PyErr_SetString(fail, "StepPlan: parameters must be plain tensors whose gradients match segs");
    return nullptr;
  }
  for (Py_ssize_t gi = 0; gi < PyList_GET_SIZE(groups); ++gi) {
    PyObject* group = PyList_GET_ITEM(groups, gi);
    PyObject* plist = PyDict_Check(group) ? PyDict_GetItem(group, k_params) : nullptr;
    if (!plist || !PyList_CheckExact(plist)) {
      Py_DECREF(self);
      PyErr_SetString(PyExc_TypeError, "StepPlan: every group needs a 'params' list");
      return nullptr;
    }
    self->group_len->push_back(PyList_GET_SIZE(plist));
  }
  return reinterpret_cast<PyObject*>(self);
}

// hyper_row(lr, beta1, beta2, eps, weight_decay, step) -> tuple of the nine
// FP32 values of the hyper set, for checking against the Python hyper_row.
PyObject* py_hyper_row(PyObject*, PyObject* args) {
  PyObject *lr, *b1, *b2, *eps, *wd;
  long long s;
  if (!PyArg_ParseTuple(args, "OOOOOL", &lr, &b1, &b2, &eps, &wd, &s)) return nullptr;
  PyObject* betas = PyTuple_Pack(2, b1, b2);
  PyObject* group = PyDict_New();
  if (!betas || !group) return nullptr;
  PyDict_SetItem(group, k_lr, lr);
  PyDict_SetItem(group, k_betas, betas);
  PyDict_SetItem(group, k_eps, eps);
  PyDict_SetItem(group, k_wd, wd);
  DfcHyper h;
  const bool ok = group_hyper(group, s, &h);
  Py_DECREF(betas);
  Py_DECREF(group);
  if (!ok) Py_RETURN_NONE;
  return Py_BuildValue("(fffffffff)", h.beta1, h.one_minus_beta1, h.beta2, h.one_minus_beta2,
                       h.sqrt_bc2, h.eps, h.decay, h.neg_step_size, h.grad_scale);
}

PyMethodDef plan_methods[] = {
    {"step", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(plan_step)), METH_FASTCALL,
     "step(stream=None) -> 1 launched, 0 plan no longer holds, <0 dfc_mt_step status"},
    {nullptr, nullptr, 0, nullptr}};

PyTypeObject PlanType = {PyVarObject_HEAD_INIT(nullptr, 0)};

PyMethodDef module_methods[] = {
    {"hyper_row", py_hyper_row, METH_VARARGS,
     "hyper_row(lr, beta1, beta2, eps, weight_decay, step) -> the FP32 hyper set"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef module_def = {PyModuleDef_HEAD_INIT, "_dfc_host",
                          "Native steady-state host path of DFCAdamW.step().", -1,
                          module_methods};

}  // namespace

PyMODINIT_FUNC PyInit__dfc_host(void) {
  PlanType.tp_name = "t3st_b200._dfc_host.StepPlan";
  PlanType.tp_basicsize = sizeof(Plan);
  PlanType.tp_flags = Py_TPFLAGS_DEFAULT | Py_TPFLAGS_HAVE_GC;
  PlanType.tp_traverse = plan_traverse;
  PlanType.tp_clear = plan_clear;
  PlanType.tp_doc = "Cached segment descriptors of DFCAdamW's steady-state step.";
  PlanType.tp_new = plan_new;
  PlanType.tp_dealloc = plan_dealloc;
  PlanType.tp_methods = plan_methods;
  if (PyType_Ready(&PlanType) < 0) return nullptr;
  k_params = PyUnicode_InternFromString("params");
  k_param_groups = PyUnicode_InternFromString("param_groups");
  k_step = PyUnicode_InternFromString("step");
  k_lr = PyUnicode_InternFromString("lr");
  k_betas = PyUnicode_InternFromString("betas");
  k_eps = PyUnicode_InternFromString("eps");
  k_wd = PyUnicode_InternFromString("weight_decay");
  if (!k_params || !k_param_groups || !k_step || !k_lr || !k_betas || !k_eps || !k_wd) return nullptr;
  PyObject* m = PyModule_Create(&module_def);
  if (!m) return nullptr;
  Py_INCREF(&PlanType);
  if (PyModule_AddObject(m, "StepPlan", reinterpret_cast<PyObject*>(&PlanType)) < 0) {
    Py_DECREF(&PlanType);
    Py_DECREF(m);
    return nullptr;
  }
  return m;
}
