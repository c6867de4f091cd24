// C ABI over the training engine (declarations and contract in distrain_c.h).
//
// The engine itself is distrain_b200.ffi_engine.FfiEngine (PyTorch shell + the sm_100a kernel library),
// so this file is a bridge: it finds or starts a Python interpreter, creates one engine object and
// forwards each call to the method of the same name, returning its JSON text in malloc'd memory.
//
// Python's C API is resolved at run time with dlsym instead of linking libpython: the interpreter that
// loads this library may carry its own statically linked copy of Python (Debian's /usr/bin/python3
// does), and a second libpython in the same process would be a second, uninitialised interpreter.
// Only functions are used (no data symbols such as Py_None), so nothing binds before that lookup.
#include <Python.h>
#include <dlfcn.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

#include "distrain_c.h"

#ifndef DT_LIBPYTHON_DEFAULT
#define DT_LIBPYTHON_DEFAULT "libpython3.12.so.1.0"
#endif
#ifndef DT_SITE_DEFAULT
#define DT_SITE_DEFAULT ""
#endif

extern "C" long long dtr_shard_assignment(const char* node_id, unsigned long long version, long long total_shards,
                                          long long shards_per_node, long long* out);

namespace {

struct PyApi {
  decltype(&Py_IsInitialized) IsInitialized;
  decltype(&Py_InitializeEx) InitializeEx;
  decltype(&PyEval_SaveThread) SaveThread;
  decltype(&PyGILState_Ensure) GILEnsure;
  decltype(&PyGILState_Release) GILRelease;
  decltype(&PyRun_SimpleStringFlags) RunString;
  decltype(&PyImport_ImportModule) Import;
  decltype(&PyObject_GetAttrString) GetAttr;
  decltype(&PyObject_CallObject) Call;
  decltype(&PyTuple_New) TupleNew;
  decltype(&PyTuple_SetItem) TupleSet;
  decltype(&PyUnicode_FromString) Str;
  decltype(&PyUnicode_AsUTF8AndSize) Utf8;
  decltype(&PyBytes_FromStringAndSize) Bytes;
  decltype(&PyFloat_FromDouble) Float;
  decltype(&PyLong_FromUnsignedLongLong) Long;
  decltype(&Py_DecRef) DecRef;
  decltype(&PyErr_Occurred) ErrOccurred;
  decltype(&PyErr_Fetch) ErrFetch;
  decltype(&PyObject_Str) ObjStr;
  decltype(&PyErr_Clear) ErrClear;
};

std::mutex g_mu;
PyApi g_py;
bool g_py_ready = false;
PyObject* g_engine = nullptr;  // FfiEngine instance (strong reference, lives until exit)
int g_use_gpu = 1;

std::string json_error(const std::string& msg) {
  std::string out = "{\"error\": \"";
  for (char c : msg) {
    if (c == '"' || c == '\\') out += '\\', out += c;
    else if (c == '\n') out += "\\n";
    else if ((unsigned char)c < 0x20) out += ' ';
    else out += c;
  }
  return out + "\"}";
}

char* dup(const std::string& s) {
  char* p = static_cast<char*>(malloc(s.size() + 1));
  if (p) memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

std::string library_dir() {
  Dl_info info;
  if (!dladdr(reinterpret_cast<void*>(&distrain_status), &info) || !info.dli_fname) return ".";
  std::string p = info.dli_fname;
  size_t k = p.rfind('/');
  return k == std::string::npos ? "." : p.substr(0, k);
}

template <class F>
bool bind(void* h, const char* name, F& slot, std::string* err) {
  slot = reinterpret_cast<F>(dlsym(h, name));
  if (!slot) *err = std::string("Python C API symbol not found: ") + name;
  return slot != nullptr;
}

std::string py_literal(const std::string& s) {  // a Python string literal of s
  std::string out = "'";
  for (char c : s) {
    if (c == '\'' || c == '\\') out += '\\';
    out += c;
  }
  return out + "'";
}

// Caller holds g_mu. Finds the process's Python or loads libpython, starts the interpreter if needed
// (releasing the GIL afterwards so every call takes it with PyGILState_Ensure).
bool ensure_python(std::string* err) {
  if (g_py_ready) return true;
  void* h = RTLD_DEFAULT;
  bool have = dlsym(RTLD_DEFAULT, "Py_IsInitialized") != nullptr;
  if (!have) {
    const char* lib = getenv("DT_LIBPYTHON");
    h = dlopen(lib && *lib ? lib : DT_LIBPYTHON_DEFAULT, RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      *err = std::string("cannot load libpython: ") + dlerror();
      return false;
    }
  }
  PyApi& a = g_py;
  if (!(bind(h, "Py_IsInitialized", a.IsInitialized, err) && bind(h, "Py_InitializeEx", a.InitializeEx, err) &&
        bind(h, "PyEval_SaveThread", a.SaveThread, err) && bind(h, "PyGILState_Ensure", a.GILEnsure, err) &&
        bind(h, "PyGILState_Release", a.GILRelease, err) && bind(h, "PyRun_SimpleStringFlags", a.RunString, err) &&
        bind(h, "PyImport_ImportModule", a.Import, err) && bind(h, "PyObject_GetAttrString", a.GetAttr, err) &&
        bind(h, "PyObject_CallObject", a.Call, err) && bind(h, "PyTuple_New", a.TupleNew, err) &&
        bind(h, "PyTuple_SetItem", a.TupleSet, err) && bind(h, "PyUnicode_FromString", a.Str, err) &&
        bind(h, "PyUnicode_AsUTF8AndSize", a.Utf8, err) && bind(h, "PyBytes_FromStringAndSize", a.Bytes, err) &&
        bind(h, "PyFloat_FromDouble", a.Float, err) && bind(h, "PyLong_FromUnsignedLongLong", a.Long, err) &&
        bind(h, "Py_DecRef", a.DecRef, err) && bind(h, "PyErr_Occurred", a.ErrOccurred, err) &&
        bind(h, "PyErr_Fetch", a.ErrFetch, err) && bind(h, "PyObject_Str", a.ObjStr, err) &&
        bind(h, "PyErr_Clear", a.ErrClear, err)))
    return false;
  bool started = false;
  if (!a.IsInitialized()) {
    a.InitializeEx(0);  // no signal handlers: the host program keeps its own
    started = true;
  }
  // module search path: the package root (two levels above this library), the site directories recorded
  // at build time (only for an interpreter started here), then DT_PYTHONPATH
  std::string lib = library_dir();
  std::string root = lib + "/../..";
  std::string code = "import sys\nfor _p in [" + py_literal(root);
  if (started) {
    std::string site = DT_SITE_DEFAULT;
    size_t b = 0;
    while (b <= site.size() && !site.empty()) {
      size_t e = site.find(':', b);
      std::string d = site.substr(b, e == std::string::npos ? std::string::npos : e - b);
      if (!d.empty()) code += ", " + py_literal(d);
      if (e == std::string::npos) break;
      b = e + 1;
    }
  }
  if (const char* extra = getenv("DT_PYTHONPATH")) {
    std::string s = extra;
    size_t b = 0;
    while (true) {
      size_t e = s.find(':', b);
      std::string d = s.substr(b, e == std::string::npos ? std::string::npos : e - b);
      if (!d.empty()) code += ", " + py_literal(d);
      if (e == std::string::npos) break;
      b = e + 1;
    }
  }
  code += "]:\n    if _p not in sys.path: sys.path.append(_p)\n";
  PyGILState_STATE st = started ? PyGILState_LOCKED : a.GILEnsure();
  int rc = a.RunString(code.c_str(), nullptr);
  if (started) a.SaveThread();  // hand the GIL back; calls take it per call
  else a.GILRelease(st);
  if (rc != 0) {
    *err = "cannot set the module search path";
    return false;
  }
  g_py_ready = true;
  return true;
}

std::string fetch_error() {
  PyObject *t = nullptr, *v = nullptr, *tb = nullptr;
  g_py.ErrFetch(&t, &v, &tb);
  std::string msg = "Python error";
  PyObject* s = v ? g_py.ObjStr(v) : (t ? g_py.ObjStr(t) : nullptr);
  if (s) {
    Py_ssize_t n = 0;
    const char* c = g_py.Utf8(s, &n);
    if (c) msg = std::string(c, n);
    g_py.DecRef(s);
  }
  g_py.ErrClear();
  if (t) g_py.DecRef(t);
  if (v) g_py.DecRef(v);
  if (tb) g_py.DecRef(tb);
  return msg;
}

// Caller holds g_mu and the GIL.
bool ensure_engine(std::string* err) {
  if (g_engine) return true;
  PyObject* mod = g_py.Import("distrain_b200.ffi_engine");
  if (!mod) {
    *err = "cannot import distrain_b200.ffi_engine: " + fetch_error();
    return false;
  }
  PyObject* cls = g_py.GetAttr(mod, "FfiEngine");
  g_py.DecRef(mod);
  if (!cls) {
    *err = fetch_error();
    return false;
  }
  g_engine = g_py.Call(cls, nullptr);
  g_py.DecRef(cls);
  if (!g_engine) {
    *err = fetch_error();
    return false;
  }
  PyObject* f = g_py.GetAttr(g_engine, "set_backend");
  PyObject* args = g_py.TupleNew(1);
  g_py.TupleSet(args, 0, g_py.Long(static_cast<unsigned long long>(g_use_gpu)));
  PyObject* r = f ? g_py.Call(f, args) : nullptr;
  g_py.DecRef(args);
  if (f) g_py.DecRef(f);
  if (!r) {
    *err = fetch_error();
    return false;
  }
  g_py.DecRef(r);
  return true;
}

// Argument builders (make_args) run with the GIL held and return a new tuple, or null on failure.
char* call(const char* method, PyObject* (*make_args)(const void*), const void* ctx) {
  std::lock_guard<std::mutex> lock(g_mu);
  std::string err;
  if (!ensure_python(&err)) return dup(json_error(err));
  PyGILState_STATE st = g_py.GILEnsure();
  std::string out;
  if (!ensure_engine(&err)) {
    out = json_error(err);
  } else {
    PyObject* f = g_py.GetAttr(g_engine, method);
    PyObject* args = make_args ? make_args(ctx) : nullptr;
    PyObject* r = (f && (args || !make_args)) ? g_py.Call(f, args) : nullptr;
    if (args) g_py.DecRef(args);
    if (f) g_py.DecRef(f);
    if (!r) {
      out = json_error(std::string(method) + ": " + fetch_error());
    } else {
      Py_ssize_t n = 0;
      const char* c = g_py.Utf8(r, &n);
      out = c ? std::string(c, n) : json_error(std::string(method) + " did not return text");
      if (!c) g_py.ErrClear();
      g_py.DecRef(r);
    }
  }
  g_py.GILRelease(st);
  return dup(out);
}

PyObject* tuple_of(int n, PyObject** items) {
  for (int i = 0; i < n; ++i)
    if (!items[i]) {
      for (int j = 0; j < n; ++j)
        if (items[j]) g_py.DecRef(items[j]);
      return nullptr;
    }
  PyObject* t = g_py.TupleNew(n);
  for (int i = 0; i < n; ++i) g_py.TupleSet(t, i, items[i]);  // steals the references
  return t;
}

PyObject* one_str(const void* ctx) {
  PyObject* it[1] = {g_py.Str(static_cast<const char*>(ctx))};
  return tuple_of(1, it);
}
PyObject* one_ull(const void* ctx) {
  PyObject* it[1] = {g_py.Long(*static_cast<const unsigned long long*>(ctx))};
  return tuple_of(1, it);
}
PyObject* one_float(const void* ctx) {
  PyObject* it[1] = {g_py.Float(*static_cast<const double*>(ctx))};
  return tuple_of(1, it);
}
struct ShardArgs {
  const char* paths;
  size_t batch, seq;
};
PyObject* shard_args(const void* ctx) {
  const ShardArgs* a = static_cast<const ShardArgs*>(ctx);
  PyObject* it[3] = {g_py.Str(a->paths), g_py.Long(a->batch), g_py.Long(a->seq)};
  return tuple_of(3, it);
}
struct BytesArgs {
  const uint8_t* data;
  size_t len;
};
PyObject* bytes_args(const void* ctx) {
  const BytesArgs* a = static_cast<const BytesArgs*>(ctx);
  PyObject* it[1] = {g_py.Bytes(reinterpret_cast<const char*>(a->data), static_cast<Py_ssize_t>(a->len))};
  return tuple_of(1, it);
}

}  // namespace

extern "C" {

void distrain_set_backend(uint8_t use_gpu) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    g_use_gpu = use_gpu ? 1 : 0;
    if (!g_engine) return;  // applied when the engine is created
  }
  unsigned long long v = use_gpu ? 1ull : 0ull;
  free(call("set_backend", one_ull, &v));
}

char* distrain_init(const char* preset) {
  if (!preset) return dup(json_error("null preset"));
  return call("init", one_str, preset);
}

char* distrain_load_shards(const char* paths_json, size_t batch_size, size_t seq_len) {
  if (!paths_json) return dup(json_error("null paths"));
  ShardArgs a{paths_json, batch_size, seq_len};
  return call("load_shards", shard_args, &a);
}

char* distrain_train_step(double learning_rate) { return call("train_step", one_float, &learning_rate); }

char* distrain_status(void) { return call("status", nullptr, nullptr); }

char* distrain_calibrate(double target_interval_secs) { return call("calibrate", one_float, &target_interval_secs); }

char* distrain_load_checkpoint_file(const char* path) {
  if (!path) return dup(json_error("null path"));
  return call("load_checkpoint_file", one_str, path);
}

char* distrain_load_checkpoint(const uint8_t* data, size_t len) {
  if (!data || len == 0) return dup(json_error("null or empty checkpoint data"));
  BytesArgs a{data, len};
  return call("load_checkpoint", bytes_args, &a);
}

char* distrain_snapshot_params(void) { return call("snapshot_params", nullptr, nullptr); }

char* distrain_compute_delta(const char* output_path) {
  if (!output_path) return dup(json_error("null output path"));
  return call("compute_delta", one_str, output_path);
}

char* distrain_default_training_params(void) { return call("default_training_params", nullptr, nullptr); }

char* distrain_compute_shard_assignment(const char* node_id, uint64_t version, uint32_t total_shards,
                                        uint32_t shards_per_node) {
  if (!node_id) return dup(json_error("null node id"));
  uint32_t n = shards_per_node < total_shards ? shards_per_node : total_shards;
  long long* out = static_cast<long long*>(malloc(sizeof(long long) * (n ? n : 1)));
  if (!out) return dup(json_error("out of memory"));
  long long k = dtr_shard_assignment(node_id, version, total_shards, shards_per_node, out);
  std::string s = "[";
  for (long long i = 0; i < k; ++i) s += (i ? ", " : "") + std::to_string(out[i]);
  free(out);
  return dup(s + "]");
}

// Linear warm-up, then cosine decay from max_lr to min_lr over the remaining steps (no clamp past
// total_steps), the schedule of the reference's cosine_lr.
double distrain_cosine_lr(uint64_t step, uint64_t warmup_steps, uint64_t total_steps, double max_lr, double min_lr) {
  if (step < warmup_steps) return max_lr * (double)step / (double)warmup_steps;
  double span = total_steps > warmup_steps ? (double)(total_steps - warmup_steps) : 1.0;
  double progress = (double)(step - warmup_steps) / span;
  return min_lr + 0.5 * (max_lr - min_lr) * (1.0 + cos(M_PI * progress));
}

// Releases the model, data and device memory of the engine. The interpreter stays: a Python runtime
// with CUDA extensions loaded is not safely finalisable, and a later distrain_init reuses it.
void distrain_shutdown(void) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_engine) return;
  }
  free(call("shutdown", nullptr, nullptr));
}

void distrain_free_string(char* ptr) { free(ptr); }

}  // extern "C"
