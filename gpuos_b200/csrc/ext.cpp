// Python module `gpuos_ext`: the reference's extension API
// (pytorch_ext/gpuos_ext.cpp:861-883) on top of the C ABI in
// include/gpuos_b200.h.  Torch is used here only to read tensor metadata and
// the current CUDA stream; all scheduling lives behind the C ABI.
//
// The submit_* entry points are METH_FASTCALL functions that read the tensors'
// pointers, shapes and strides directly (a few hundred nanoseconds per call).
// Errors raise RuntimeError / ValueError / TypeError instead of exiting the
// process.
#include <Python.h>

#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>

#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gpuos_b200.h"

namespace {

constexpr int kMaxDev = 64;
gpuos_executor* g_ex[kMaxDev] = {nullptr};
gpuos_options g_opt;
bool g_have_opt = false;
int g_verbose = 0;
std::mutex g_mu;

// Tensors of submitted requests stay referenced until the batch that reads
// them is done, so that dropping the Python objects (or the caching allocator
// handing their memory to a new tensor) cannot corrupt a pending request.
// All of this runs with the GIL held.
struct Keep {
  uint64_t ticket;
  std::vector<PyObject*> objs;
};
std::vector<PyObject*> g_pending_refs[kMaxDev];
std::deque<Keep> g_inflight_refs[kMaxDev];

inline void keep(int dev, PyObject* o) {
  Py_INCREF(o);
  g_pending_refs[dev].push_back(o);
}

void release_done(int dev, bool all) {
  auto& q = g_inflight_refs[dev];
  uint64_t done = UINT64_MAX;
  if (!all) {
    gpuos_stats st;
    if (!g_ex[dev] || gpuos_get_stats(g_ex[dev], &st) != GPUOS_OK) return;
    done = st.processed;
  }
  while (!q.empty() && q.front().ticket <= done) {
    for (PyObject* o : q.front().objs) Py_DECREF(o);
    q.pop_front();
  }
  if (all) {
    for (PyObject* o : g_pending_refs[dev]) Py_DECREF(o);
    g_pending_refs[dev].clear();
  }
}

PyObject* raise_status(int32_t rc) {
  const char* msg = gpuos_last_error();
  PyObject* type = PyExc_RuntimeError;
  if (rc == GPUOS_EINVAL) type = PyExc_ValueError;
  PyErr_SetString(type, (msg && *msg) ? msg : "gpuos error");
  return nullptr;
}

bool fill_desc(PyObject* obj, gpuos_tensor* d, int* dev, const char* name) {
  if (!THPVariable_Check(obj)) {
    PyErr_Format(PyExc_TypeError, "%s must be a torch.Tensor", name);
    return false;
  }
  const at::Tensor& t = THPVariable_Unpack(obj);
  if (!t.is_cuda()) {
    PyErr_Format(PyExc_RuntimeError, "tensors must be CUDA (%s is on %s)", name,
                 t.device().str().c_str());
    return false;
  }
  switch (t.scalar_type()) {
    case at::kFloat: d->dtype = GPUOS_F32; break;
    case at::kHalf: d->dtype = GPUOS_F16; break;
    case at::kBFloat16: d->dtype = GPUOS_BF16; break;
    default:
      PyErr_Format(PyExc_TypeError, "%s: dtype %s is not supported (float32, float16, bfloat16)",
                   name, std::string(c10::toString(t.scalar_type())).c_str());
      return false;
  }
  const int64_t nd = t.dim();
  if (nd > 8) {
    PyErr_Format(PyExc_ValueError, "%s has %lld dims; at most 8 are supported", name,
                 (long long)nd);
    return false;
  }
  d->ndim = (int32_t)nd;
  d->data = t.numel() ? const_cast<void*>(t.const_data_ptr()) : nullptr;
  const auto sz = t.sizes();
  const auto st = t.strides();
  for (int64_t i = 0; i < nd; ++i) {
    d->sizes[i] = sz[i];
    d->strides[i] = st[i];
  }
  *dev = t.get_device();
  return true;
}

gpuos_executor* executor_for(int dev) {
  if (dev < 0 || dev >= kMaxDev) {
    PyErr_SetString(PyExc_RuntimeError, "device index out of range");
    return nullptr;
  }
  if (g_ex[dev]) return g_ex[dev];
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_ex[dev]) return g_ex[dev];
  if (!g_have_opt) {
    PyErr_SetString(PyExc_RuntimeError, "gpuos not initialized");
    return nullptr;
  }
  gpuos_executor* ex = nullptr;
  int32_t rc;
  Py_BEGIN_ALLOW_THREADS rc = gpuos_executor_create(dev, &g_opt, &ex);
  Py_END_ALLOW_THREADS if (rc != GPUOS_OK) {
    raise_status(rc);
    return nullptr;
  }
  g_ex[dev] = ex;
  return ex;
}

// current CUDA device; -1 with a Python error set when CUDA is unusable
int current_device() {
  try {
    return (int)c10::cuda::current_device();
  } catch (const std::exception& e) {
    PyErr_Format(PyExc_RuntimeError, "CUDA is not available: %s", e.what());
    return -1;
  }
}

bool current_stream(int dev, cudaStream_t* s) {
  try {
    *s = c10::cuda::getCurrentCUDAStream((c10::DeviceIndex)dev).stream();
    return true;
  } catch (const std::exception& e) {
    PyErr_Format(PyExc_RuntimeError, "CUDA is not available: %s", e.what());
    return false;
  }
}

// ---- lifecycle ---------------------------------------------------------------
PyObject* py_init(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwl[] = {"capacity", "threads_per_block", "mode", "blocks_per_sm",
                              "idle_ms", "max_batch", nullptr};
  int capacity = 4096, tpb = 256, bps = 0, max_batch = 0;
  double idle_ms = 0.0;
  const char* mode = nullptr;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|iizidi", const_cast<char**>(kwl), &capacity, &tpb,
                                   &mode, &bps, &idle_ms, &max_batch))
    return nullptr;
  if (!mode || !*mode) {
    const char* env = std::getenv("GPUOS_MODE");
    mode = (env && *env) ? env : "persistent";
  }
  int m;
  if (!std::strcmp(mode, "persistent")) m = GPUOS_MODE_PERSISTENT;
  else if (!std::strcmp(mode, "stream")) m = GPUOS_MODE_STREAM;
  else {
    PyErr_SetString(PyExc_ValueError, "mode must be 'persistent' or 'stream'");
    return nullptr;
  }
  const int dev = current_device();
  if (dev < 0) return nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_ex[dev]) Py_RETURN_NONE;  // already started (reference: init is idempotent)
    std::memset(&g_opt, 0, sizeof(g_opt));
    g_opt.capacity = capacity;
    g_opt.threads_per_block = tpb;
    g_opt.mode = m;
    g_opt.blocks_per_sm = bps;
    g_opt.idle_ms = idle_ms;
    g_opt.max_batch = max_batch;
    g_have_opt = true;
  }
  if (!executor_for(dev)) return nullptr;
  Py_RETURN_NONE;
}

PyObject* py_shutdown(PyObject*, PyObject*) {
  std::string err;
  int32_t first_rc = GPUOS_OK;
  for (int d = 0; d < kMaxDev; ++d) {
    gpuos_executor* ex = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      ex = g_ex[d];
      g_ex[d] = nullptr;
    }
    if (!ex) continue;
    int32_t rc;
    Py_BEGIN_ALLOW_THREADS rc = gpuos_executor_destroy(ex);
    Py_END_ALLOW_THREADS if (rc != GPUOS_OK && first_rc == GPUOS_OK) {
      first_rc = rc;
      err = gpuos_last_error();
    }
    release_done(d, true);
  }
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_have_opt = false;
  }
  if (first_rc != GPUOS_OK) {
    PyErr_SetString(PyExc_RuntimeError, err.c_str());
    return nullptr;
  }
  Py_RETURN_NONE;
}

PyObject* py_abi_version(PyObject*, PyObject*) { return PyLong_FromLong(gpuos_abi_version()); }

PyObject* py_set_debug_level(PyObject*, PyObject* arg) {
  const long lvl = PyLong_AsLong(arg);
  if (PyErr_Occurred()) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d]) {
      const int32_t rc = gpuos_set_debug_level(g_ex[d], (int32_t)lvl);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  Py_RETURN_NONE;
}

PyObject* py_set_verbose_level(PyObject*, PyObject* arg) {
  const long lvl = PyLong_AsLong(arg);
  if (PyErr_Occurred()) return nullptr;
  g_verbose = (int)lvl;
  Py_RETURN_NONE;
}

PyObject* py_set_yield_every(PyObject*, PyObject* arg) {
  const unsigned long long n = PyLong_AsUnsignedLongLong(arg);
  if (PyErr_Occurred()) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d]) {
      const int32_t rc = gpuos_set_yield_every(g_ex[d], n);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  Py_RETURN_NONE;
}

PyObject* py_worker_alive(PyObject*, PyObject*) {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  if (dev >= kMaxDev || !g_ex[dev]) Py_RETURN_FALSE;
  const int32_t rc = gpuos_worker_alive(g_ex[dev]);
  if (rc < 0) return raise_status(rc);
  if (rc) Py_RETURN_TRUE;
  Py_RETURN_FALSE;
}

PyObject* stats_dict(const gpuos_stats& s, bool reference_keys_only) {
  PyObject* d = PyDict_New();
  auto put = [&](const char* k, PyObject* v) {
    PyDict_SetItemString(d, k, v);
    Py_DECREF(v);
  };
  const uint64_t inflight = s.published >= s.processed ? s.published - s.processed : 0;
  put("head", PyLong_FromUnsignedLongLong(s.staged));
  put("tail", PyLong_FromUnsignedLongLong(s.published));
  put("in_flight", PyLong_FromUnsignedLongLong(inflight));
  put("capacity", PyLong_FromLong(s.capacity));
  put("processed", PyLong_FromUnsignedLongLong(s.processed));
  put("heartbeat", PyLong_FromUnsignedLongLong(s.heartbeat));
  put("quit", PyLong_FromLong(s.quit));
  put("host_tail_shadow", PyLong_FromUnsignedLongLong(s.published));
  put("host_pending", PyLong_FromUnsignedLongLong(s.pending));
  put("staging", PyUnicode_FromString(s.mode == GPUOS_MODE_PERSISTENT ? "mapped" : "stream"));
  put("shard_size", PyLong_FromLong(s.max_batch));
  if (!reference_keys_only) {
    put("mode", PyUnicode_FromString(s.mode == GPUOS_MODE_PERSISTENT ? "persistent" : "stream"));
    put("retired", PyLong_FromUnsignedLongLong(s.retired));
    put("requests", PyLong_FromUnsignedLongLong(s.requests));
    put("errors", PyLong_FromUnsignedLongLong(s.errors));
    put("relaunches", PyLong_FromUnsignedLongLong(s.relaunches));
    put("dev_ns", PyLong_FromUnsignedLongLong(s.dev_ns));
    put("lean", PyLong_FromUnsignedLongLong(s.lean));
    put("chain", PyLong_FromUnsignedLongLong(s.chain));
    put("worker_alive", PyBool_FromLong(s.worker_alive));
    put("grid", PyLong_FromLong(s.grid));
    put("block", PyLong_FromLong(s.block));
    put("device", PyLong_FromLong(s.device));
  }
  return d;
}

PyObject* py_peek_queue(PyObject*, PyObject*) {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  if (dev >= kMaxDev || !g_ex[dev]) {
    PyErr_SetString(PyExc_RuntimeError, "gpuos not initialized");
    return nullptr;
  }
  gpuos_stats s;
  const int32_t rc = gpuos_get_stats(g_ex[dev], &s);
  if (rc != GPUOS_OK) return raise_status(rc);
  return stats_dict(s, false);
}

// ---- submission ------------------------------------------------------------
PyObject* submit_builtin(int op, PyObject* const* args, Py_ssize_t n) {
  if (n != 3) {
    PyErr_SetString(PyExc_TypeError, "expected (a, b, out)");
    return nullptr;
  }
  gpuos_tensor a, b, o;
  int da, db, dout;
  if (!fill_desc(args[0], &a, &da, "a") || !fill_desc(args[1], &b, &db, "b") ||
      !fill_desc(args[2], &o, &dout, "out"))
    return nullptr;
  if (da != dout || db != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  gpuos_executor* ex = executor_for(dout);
  if (!ex) return nullptr;
  const int32_t rc = gpuos_submit_builtin(ex, op, &a, &b, &o);
  if (rc != GPUOS_OK) return raise_status(rc);
  keep(dout, args[0]);
  keep(dout, args[1]);
  keep(dout, args[2]);
  Py_RETURN_NONE;
}

PyObject* py_submit_add(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_builtin(GPUOS_OP_ADD, a, n); }
PyObject* py_submit_mul(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_builtin(GPUOS_OP_MUL, a, n); }
PyObject* py_submit_sub(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_builtin(GPUOS_OP_SUB, a, n); }
PyObject* py_submit_div(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_builtin(GPUOS_OP_DIV, a, n); }

PyObject* py_submit_unary(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 3) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, a, out)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (PyErr_Occurred()) return nullptr;
  gpuos_tensor a, o;
  int da, dout;
  if (!fill_desc(args[1], &a, &da, "a") || !fill_desc(args[2], &o, &dout, "out")) return nullptr;
  if (da != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  gpuos_executor* ex = executor_for(dout);
  if (!ex) return nullptr;
  const int32_t rc = gpuos_submit_unary(ex, (int32_t)slot, &a, &o);
  if (rc != GPUOS_OK) return raise_status(rc);
  keep(dout, args[1]);
  keep(dout, args[2]);
  Py_RETURN_NONE;
}

PyObject* py_submit_binary(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 4) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, a, b, out)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (PyErr_Occurred()) return nullptr;
  gpuos_tensor a, b, o;
  int da, db, dout;
  if (!fill_desc(args[1], &a, &da, "a") || !fill_desc(args[2], &b, &db, "b") ||
      !fill_desc(args[3], &o, &dout, "out"))
    return nullptr;
  if (da != dout || db != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  gpuos_executor* ex = executor_for(dout);
  if (!ex) return nullptr;
  const int32_t rc = gpuos_submit_binary(ex, (int32_t)slot, &a, &b, &o);
  if (rc != GPUOS_OK) return raise_status(rc);
  keep(dout, args[1]);
  keep(dout, args[2]);
  keep(dout, args[3]);
  Py_RETURN_NONE;
}

// submit_nary(slot, inputs, out): a custom expression of 1 to 4 inputs (no
// counterpart in the reference module, whose requests take two at most).
PyObject* py_submit_nary(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 3) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, inputs, out)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (PyErr_Occurred()) return nullptr;
  PyObject* seq = PySequence_Fast(args[1], "inputs must be a sequence of tensors");
  if (!seq) return nullptr;
  const Py_ssize_t nin = PySequence_Fast_GET_SIZE(seq);
  if (nin < 1 || nin > 4) {
    Py_DECREF(seq);
    PyErr_SetString(PyExc_ValueError, "a request takes 1 to 4 inputs");
    return nullptr;
  }
  gpuos_tensor ins[4], o;
  int dout;
  if (!fill_desc(args[2], &o, &dout, "out")) {
    Py_DECREF(seq);
    return nullptr;
  }
  static const char* names[4] = {"a", "b", "c", "d"};
  for (Py_ssize_t k = 0; k < nin; ++k) {
    int d;
    if (!fill_desc(PySequence_Fast_GET_ITEM(seq, k), &ins[k], &d, names[k])) {
      Py_DECREF(seq);
      return nullptr;
    }
    if (d != dout) {
      Py_DECREF(seq);
      PyErr_SetString(PyExc_RuntimeError, "device mismatch");
      return nullptr;
    }
  }
  gpuos_executor* ex = executor_for(dout);
  if (!ex) {
    Py_DECREF(seq);
    return nullptr;
  }
  const int32_t rc = gpuos_submit_nary(ex, (int32_t)slot, (int32_t)nin, ins, &o);
  if (rc != GPUOS_OK) {
    Py_DECREF(seq);
    return raise_status(rc);
  }
  for (Py_ssize_t k = 0; k < nin; ++k) keep(dout, PySequence_Fast_GET_ITEM(seq, k));
  keep(dout, args[2]);
  Py_DECREF(seq);
  Py_RETURN_NONE;
}

PyObject* py_submit_reduce(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 5) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, x, out, axes, keepdim)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (PyErr_Occurred()) return nullptr;
  gpuos_tensor x, o;
  int dx, dout;
  if (!fill_desc(args[1], &x, &dx, "x") || !fill_desc(args[2], &o, &dout, "out")) return nullptr;
  if (dx != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  PyObject* seq = PySequence_Fast(args[3], "axes must be a sequence of ints");
  if (!seq) return nullptr;
  const Py_ssize_t na = PySequence_Fast_GET_SIZE(seq);
  if (na > 8) {
    Py_DECREF(seq);
    PyErr_SetString(PyExc_ValueError, "at most 8 axes");
    return nullptr;
  }
  int32_t axes[8];
  for (Py_ssize_t i = 0; i < na; ++i) {
    axes[i] = (int32_t)PyLong_AsLong(PySequence_Fast_GET_ITEM(seq, i));
  }
  Py_DECREF(seq);
  if (PyErr_Occurred()) return nullptr;
  const int keepdim = PyObject_IsTrue(args[4]);
  if (keepdim < 0) return nullptr;
  gpuos_executor* ex = executor_for(dout);
  if (!ex) return nullptr;
  const int32_t rc = gpuos_submit_reduce(ex, (int32_t)slot, &x, &o, axes, (int32_t)na, keepdim);
  if (rc != GPUOS_OK) return raise_status(rc);
  keep(dout, args[1]);
  keep(dout, args[2]);
  Py_RETURN_NONE;
}

// ---- flush -----------------------------------------------------------------
PyObject* py_flush(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwl[] = {"sync", nullptr};
  int sync = 0;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|p", const_cast<char**>(kwl), &sync)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d) {
    gpuos_executor* ex = g_ex[d];
    if (!ex) continue;
    cudaStream_t s = nullptr;
    if (!current_stream(d, &s)) return nullptr;
    int32_t rc;
    uint64_t ticket = 0;
    Py_BEGIN_ALLOW_THREADS rc = gpuos_flush(ex, sync, s, &ticket);
    Py_END_ALLOW_THREADS if (rc != GPUOS_OK) return raise_status(rc);
    if (!g_pending_refs[d].empty()) {
      g_inflight_refs[d].push_back(Keep{ticket, std::move(g_pending_refs[d])});
      g_pending_refs[d].clear();
    }
    release_done(d, false);
  }
  Py_RETURN_NONE;
}

// ---- jump table ----------------------------------------------------------------
gpuos_executor* current_executor() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  return executor_for(dev);
}

PyObject* py_register_elementwise(PyObject*, PyObject* args) {
  const char *key, *expr;
  int arity;
  if (!PyArg_ParseTuple(args, "ssi", &key, &expr, &arity)) return nullptr;
  gpuos_executor* ex = current_executor();
  if (!ex) return nullptr;
  int32_t slot = -1, rc;
  Py_BEGIN_ALLOW_THREADS rc = gpuos_register_elementwise(ex, key, expr, arity, &slot);
  Py_END_ALLOW_THREADS if (rc != GPUOS_OK) return raise_status(rc);
  // keep the slot numbering identical on every device already running
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d] && g_ex[d] != ex) {
      int32_t s2 = -1;
      rc = gpuos_register_elementwise(g_ex[d], key, expr, arity, &s2);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  return PyLong_FromLong(slot);
}

PyObject* py_register_reduce(PyObject*, PyObject* args) {
  const char *key, *op;
  if (!PyArg_ParseTuple(args, "ss", &key, &op)) return nullptr;
  gpuos_executor* ex = current_executor();
  if (!ex) return nullptr;
  int32_t slot = -1;
  int32_t rc = gpuos_register_reduce(ex, key, op, &slot);
  if (rc != GPUOS_OK) return raise_status(rc);
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d] && g_ex[d] != ex) {
      int32_t s2 = -1;
      rc = gpuos_register_reduce(g_ex[d], key, op, &s2);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  return PyLong_FromLong(slot);
}

PyObject* py_set_alias(PyObject*, PyObject* args) {
  int logical, physical;
  if (!PyArg_ParseTuple(args, "ii", &logical, &physical)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d]) {
      const int32_t rc = gpuos_set_alias(g_ex[d], logical, physical);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  Py_RETURN_NONE;
}

PyObject* py_set_slot(PyObject*, PyObject* args) {
  int slot;
  const char* name;
  float p0 = 0.f, p1 = 0.f;
  if (!PyArg_ParseTuple(args, "is|ff", &slot, &name, &p0, &p1)) return nullptr;
  const int v = gpuos_variant_by_name(name);
  if (v < 0) {
    PyErr_Format(PyExc_ValueError, "unknown operator name '%s'", name);
    return nullptr;
  }
  for (int d = 0; d < kMaxDev; ++d)
    if (g_ex[d]) {
      const int32_t rc = gpuos_set_slot(g_ex[d], slot, v, p0, p1);
      if (rc != GPUOS_OK) return raise_status(rc);
    }
  Py_RETURN_NONE;
}

PyObject* py_get_slot(PyObject*, PyObject* args) {
  int slot;
  if (!PyArg_ParseTuple(args, "i", &slot)) return nullptr;
  gpuos_executor* ex = current_executor();
  if (!ex) return nullptr;
  int32_t v = 0, al = 0;
  float p0 = 0, p1 = 0;
  const int32_t rc = gpuos_get_slot(ex, slot, &v, &p0, &p1, &al);
  if (rc != GPUOS_OK) return raise_status(rc);
  return Py_BuildValue("{s:i,s:f,s:f,s:i}", "variant", v, "p0", p0, "p1", p1, "alias", al);
}

PyObject* py_variant_id(PyObject*, PyObject* arg) {
  const char* name = PyUnicode_AsUTF8(arg);
  if (!name) return nullptr;
  return PyLong_FromLong(gpuos_variant_by_name(name));
}

PyMethodDef kMethods[] = {
    {"init", (PyCFunction)(void (*)(void))py_init, METH_VARARGS | METH_KEYWORDS,
     "init(capacity=4096, threads_per_block=256, mode=None, blocks_per_sm=0, idle_ms=0, "
     "max_batch=0): start the executor on the current device"},
    {"shutdown", py_shutdown, METH_NOARGS, "drain every executor and stop it"},
    {"abi_version", py_abi_version, METH_NOARGS, "ABI version (1)"},
    {"set_debug_level", py_set_debug_level, METH_O, "set device debug level"},
    {"set_verbose_level", py_set_verbose_level, METH_O, "set host verbose level"},
    {"peek_queue", py_peek_queue, METH_NOARGS, "queue and worker counters of the current device"},
    {"set_yield_every", py_set_yield_every, METH_O,
     "persistent worker exits after every N batches (0 = never)"},
    {"worker_alive", py_worker_alive, METH_NOARGS, "True while the persistent worker runs"},
    {"submit_add", (PyCFunction)(void (*)(void))py_submit_add, METH_FASTCALL, "queue out = a + b"},
    {"submit_mul", (PyCFunction)(void (*)(void))py_submit_mul, METH_FASTCALL, "queue out = a * b"},
    {"submit_sub", (PyCFunction)(void (*)(void))py_submit_sub, METH_FASTCALL, "queue out = a - b"},
    {"submit_div", (PyCFunction)(void (*)(void))py_submit_div, METH_FASTCALL,
     "queue out = a / b (0 where b == 0)"},
    {"flush", (PyCFunction)(void (*)(void))py_flush, METH_VARARGS | METH_KEYWORDS,
     "flush(sync=False): publish queued requests"},
    {"register_elementwise", py_register_elementwise, METH_VARARGS,
     "register_elementwise(key, expr, arity) -> slot"},
    {"submit_unary", (PyCFunction)(void (*)(void))py_submit_unary, METH_FASTCALL,
     "submit_unary(slot, a, out)"},
    {"submit_binary", (PyCFunction)(void (*)(void))py_submit_binary, METH_FASTCALL,
     "submit_binary(slot, a, b, out)"},
    {"submit_nary", (PyCFunction)(void (*)(void))py_submit_nary, METH_FASTCALL,
     "submit_nary(slot, inputs, out): a custom expression of 1 to 4 inputs"},
    {"register_reduce", py_register_reduce, METH_VARARGS, "register_reduce(key, 'sum'|'mean') -> slot"},
    {"submit_reduce", (PyCFunction)(void (*)(void))py_submit_reduce, METH_FASTCALL,
     "submit_reduce(slot, x, out, axes, keepdim)"},
    {"set_alias", py_set_alias, METH_VARARGS, "set_alias(logical, physical): dual-slot switch"},
    {"set_slot", py_set_slot, METH_VARARGS, "set_slot(slot, op_name, p0=0, p1=0): online switch"},
    {"get_slot", py_get_slot, METH_VARARGS, "get_slot(slot) -> dict"},
    {"variant_id", py_variant_id, METH_O, "operator id of a builtin name, or -1"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "gpuos_ext",
                       "B200 aggregated small-op executor (reference-compatible API)", -1,
                       kMethods};

}  // namespace

PyMODINIT_FUNC PyInit_gpuos_ext(void) { return PyModule_Create(&kModule); }
