"""Build libcra.so in-tree with nvcc for sm_100a.

    python cron-root-attention_b200/build.py [--force]

Compiles every ``csrc/*.cu`` to an object (skipped when up to date) and links
them into ``cron_root_attention/libcra.so`` (CUDA runtime linked statically;
the driver is reached through cudaGetDriverEntryPoint, so no -lcuda).
Also builds the test-only ``cron_root_attention/libcra_waitprobe.so`` from
``csrc/testing/wait_probe.cu`` with a 0.2 ms wait limit (used by the failure
handling tests, never by the package).
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "cron_root_attention", "libcra.so")
PROBE_SRC = os.path.join(CSRC, "testing", "wait_probe.cu")
PROBE_OUT = os.path.join(HERE, "cron_root_attention", "libcra_waitprobe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def _newer(src_files, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_files)


def build(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(HERE, "..", "include", "cra.h")]
    objs = []
    for cu in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        o = os.path.join(OBJ, os.path.basename(cu)[:-3] + ".o")
        if force or _newer([cu] + headers, o):
            cmd = [NVCC] + FLAGS + ["-c", cu, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
        objs.append(o)
    if force or _newer(objs, OUT):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", OUT] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    if force or _newer([PROBE_SRC] + headers, PROBE_OUT):
        cmd = [NVCC] + FLAGS + ["-DCRA_WAIT_LIMIT_NS=200000ull", "-shared", PROBE_SRC, "-o", PROBE_OUT]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
