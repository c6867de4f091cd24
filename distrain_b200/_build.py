"""In-tree native build: CUDA kernel library (sm_100a) and C++ runtime library.

* ``csrc/kernels/*.cu``  -> ``distrain_b200/lib/libdt_kernels.so``  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``)
* ``csrc/runtime/*.cpp`` -> ``distrain_b200/lib/libdt_runtime.so``  (g++, C++17, POSIX threads/sockets)

Kernels are compiled as relocatable device code (``-rdc=true``) so the library-wide device error
word defined in ``errors.cu`` is one object shared by every kernel. Objects are compiled in parallel into ``_build/`` and relinked only when a source or header changed.
Neither library includes torch headers: they export a plain C ABI that Python binds with ctypes, so a
kernel edit rebuilds in seconds and the same ``.so`` serves non-Python callers.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "csrc")
LIBDIR = os.path.join(ROOT, "distrain_b200", "lib")
BUILDDIR = os.path.join(ROOT, "_build")

KERNELS_SO = os.path.join(LIBDIR, "libdt_kernels.so")
RUNTIME_SO = os.path.join(LIBDIR, "libdt_runtime.so")
FFI_SO = os.path.join(LIBDIR, "libdistrain_c.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA kernel library cannot be built")


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


class _BuildLock:
    """Exclusive lock on ``_build/.lock`` for one build step: the ranks of a multi-process launch that find
    the libraries stale build them one at a time (the first builds, the others then find them current)
    instead of racing on the same object and output files."""

    def __enter__(self):
        import fcntl
        os.makedirs(BUILDDIR, exist_ok=True)
        self.f = open(os.path.join(BUILDDIR, ".lock"), "w")
        fcntl.flock(self.f, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        import fcntl
        fcntl.flock(self.f, fcntl.LOCK_UN)
        self.f.close()


def _compile_many(jobs, workers):
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        futs = [ex.submit(_run, j) for j in jobs]
        for f in futs:
            f.result()


def _build_kernels(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    hdrs = glob.glob(os.path.join(CSRC, "kernels", "*.cuh")) + glob.glob(os.path.join(CSRC, "kernels", "*.h"))
    os.makedirs(LIBDIR, exist_ok=True)
    odir = os.path.join(BUILDDIR, "kernels")
    os.makedirs(odir, exist_ok=True)
    nvcc = _nvcc()
    flags = ARCH_FLAGS + ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
                          "--expt-relaxed-constexpr",
                          "-I", os.path.join(CSRC, "kernels")] + list(extra_flags or [])
    if os.environ.get("DT_BOUNDS_CHECK"):
        flags.append("-DDT_BOUNDS_CHECK=1")
    hdr_time = _newest(hdrs + [__file__])
    jobs, objs = [], []
    for s in srcs:
        o = os.path.join(odir, os.path.basename(s) + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            jobs.append([nvcc] + flags + ["-c", s, "-o", o])
    if jobs:
        if verbose:
            print(f"[build] nvcc {len(jobs)} kernel sources", file=sys.stderr)
        _compile_many(jobs, min(len(jobs), os.cpu_count() or 4))
    if jobs or force or not os.path.exists(KERNELS_SO) or os.path.getmtime(KERNELS_SO) < _newest(objs):
        tmp = f"{KERNELS_SO}.{os.getpid()}.tmp"
        _run([nvcc] + ARCH_FLAGS + ["-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o", tmp] + objs)
        os.replace(tmp, KERNELS_SO)
    return KERNELS_SO


def _build_runtime(force: bool = False, verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "runtime", "*.cpp")))
    hdrs = glob.glob(os.path.join(CSRC, "runtime", "*.h")) + glob.glob(os.path.join(CSRC, "runtime", "*.hpp"))
    os.makedirs(LIBDIR, exist_ok=True)
    odir = os.path.join(BUILDDIR, "runtime")
    os.makedirs(odir, exist_ok=True)
    cxx = os.environ.get("CXX", "g++")
    flags = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function", "-pthread",
             "-I", os.path.join(CSRC, "runtime")]
    if os.environ.get("DT_SANITIZE"):
        flags += ["-fsanitize=" + os.environ["DT_SANITIZE"], "-g", "-O1"]
    hdr_time = _newest(hdrs + [__file__])
    jobs, objs = [], []
    for s in srcs:
        o = os.path.join(odir, os.path.basename(s) + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            jobs.append([cxx] + flags + ["-c", s, "-o", o])
    if not srcs:
        return ""
    if jobs:
        if verbose:
            print(f"[build] g++ {len(jobs)} runtime sources", file=sys.stderr)
        _compile_many(jobs, min(len(jobs), os.cpu_count() or 4))
    if jobs or force or not os.path.exists(RUNTIME_SO) or os.path.getmtime(RUNTIME_SO) < _newest(objs):
        tmp = f"{RUNTIME_SO}.{os.getpid()}.tmp"
        link = [cxx, "-shared", "-pthread", "-o", tmp] + objs + ["-ldl"]
        if os.environ.get("DT_SANITIZE"):
            link.insert(1, "-fsanitize=" + os.environ["DT_SANITIZE"])
        _run(link)
        os.replace(tmp, RUNTIME_SO)
    return RUNTIME_SO


def build_kernels(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    with _BuildLock():
        return _build_kernels(force, verbose, extra_flags)


def build_runtime(force: bool = False, verbose: bool = False) -> str:
    with _BuildLock():
        return _build_runtime(force, verbose)


def build_ffi(force: bool = False, verbose: bool = False) -> str:
    """``csrc/ffi/distrain_c.cpp`` -> ``libdistrain_c.so``: the C ABI over the training engine. It links
    the runtime library (native shard assignment) and resolves Python's C API at run time; the default
    libpython and the interpreter's site directories are recorded for C programs that start Python
    through it."""
    import site
    import sysconfig
    src = os.path.join(CSRC, "ffi", "distrain_c.cpp")
    if not os.path.exists(src):
        return ""
    runtime = build_runtime(force=False, verbose=verbose)
    deps = [src, os.path.join(CSRC, "ffi", "distrain_c.h"), runtime, __file__]
    if not force and os.path.exists(FFI_SO) and os.path.getmtime(FFI_SO) >= _newest(deps):
        return FFI_SO
    libpy = os.path.join(sysconfig.get_config_var("LIBDIR") or "", sysconfig.get_config_var("INSTSONAME") or "")
    sites = ":".join(p for p in site.getsitepackages() if os.path.isdir(p))
    cxx = os.environ.get("CXX", "g++")
    tmp = FFI_SO + ".tmp"
    _run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I", sysconfig.get_paths()["include"],
          f'-DDT_LIBPYTHON_DEFAULT="{libpy}"', f'-DDT_SITE_DEFAULT="{sites}"', src, "-o", tmp,
          "-L", LIBDIR, "-ldt_runtime", "-Wl,-rpath,$ORIGIN", "-ldl"])
    os.replace(tmp, FFI_SO)
    if verbose:
        print("[build] g++ C ABI library", file=sys.stderr)
    return FFI_SO


def sanitizer_cxx(sanitize: str):
    """The first of $CXX and g++ that compiles and links a program with -fsanitize=<sanitize> (None if
    neither does: a toolchain without the sanitizer runtime libraries)."""
    seen = []
    for c in (os.environ.get("CXX"), "g++"):
        if not c or c in seen:
            continue
        seen.append(c)
        try:
            r = subprocess.run([c, "-fsanitize=" + sanitize, "-x", "c++", "-", "-o", os.devnull],
                               input=b"int main(){return 0;}", capture_output=True, timeout=120)
        except (OSError, subprocess.TimeoutExpired):
            continue
        if r.returncode == 0:
            return c
    return None


def build_runtime_selftest(sanitize: str, tag: str) -> str:
    """The runtime sources plus ``csrc/runtime/tests/selftest.cpp`` as one executable built with
    ``-fsanitize=<sanitize>`` (e.g. "address,undefined" or "thread"); returns its path."""
    srcs = sorted(glob.glob(os.path.join(CSRC, "runtime", "*.cpp"))) + [os.path.join(CSRC, "runtime", "tests",
                                                                                     "selftest.cpp")]
    hdrs = glob.glob(os.path.join(CSRC, "runtime", "*.hpp")) + glob.glob(os.path.join(CSRC, "runtime", "*.h"))
    odir = os.path.join(BUILDDIR, "selftest-" + tag)
    os.makedirs(odir, exist_ok=True)
    cxx = sanitizer_cxx(sanitize)
    if cxx is None:
        raise RuntimeError(f"no C++ compiler here links -fsanitize={sanitize}")
    flags = ["-O1", "-g", "-std=c++17", "-pthread", "-fno-omit-frame-pointer", "-fsanitize=" + sanitize,
             "-I", os.path.join(CSRC, "runtime")]
    hdr_time = _newest(hdrs + [__file__])
    jobs, objs = [], []
    for src in srcs:
        o = os.path.join(odir, os.path.basename(src) + ".o")
        objs.append(o)
        if not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(src), hdr_time):
            jobs.append([cxx] + flags + ["-c", src, "-o", o])
    if jobs:
        _compile_many(jobs, min(len(jobs), os.cpu_count() or 4))
    exe = os.path.join(odir, "selftest")
    if jobs or not os.path.exists(exe) or os.path.getmtime(exe) < _newest(objs):
        _run([cxx, "-fsanitize=" + sanitize, "-pthread", "-o", exe] + objs + ["-ldl"])
    return exe


def kernels_stale() -> bool:
    srcs = glob.glob(os.path.join(CSRC, "kernels", "*.cu")) + glob.glob(os.path.join(CSRC, "kernels", "*.cuh"))
    return not os.path.exists(KERNELS_SO) or os.path.getmtime(KERNELS_SO) < _newest(srcs)


def runtime_stale() -> bool:
    srcs = glob.glob(os.path.join(CSRC, "runtime", "*.cpp")) + glob.glob(os.path.join(CSRC, "runtime", "*.h"))
    return bool(srcs) and (not os.path.exists(RUNTIME_SO) or os.path.getmtime(RUNTIME_SO) < _newest(srcs))


def build_all(force: bool = False, verbose: bool = True):
    with cf.ThreadPoolExecutor(max_workers=2) as ex:
        a = ex.submit(build_kernels, force, verbose)
        b = ex.submit(build_runtime, force, verbose)
        kernels, runtime = a.result(), b.result()
    return kernels, runtime, build_ffi(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(KERNELS_SO, RUNTIME_SO, FFI_SO)
