"""Build libq3attn.so in-tree for sm_100a (B200) with nvcc.

    python -m q3attn.build            (from qwen3-tts-engine_b200/)   or   q3attn.build.build()

Every .cu under qwen3-tts-engine_b200/csrc is compiled separately (in parallel) and linked into
qwen3-tts-engine_b200/q3attn/libq3attn.so next to this file, where q3attn._lib loads it. Objects go to
qwen3-tts-engine_b200/_build/. A rebuild happens only when a source or header is newer than the library.
"""
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                       # qwen3-tts-engine_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libq3attn.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", CSRC, "-I", INCLUDE] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the q3attn CUDA library cannot be built")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and not ptxas_info and up_to_date():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src):
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, "-c", src, "-o", obj] + NVCC_FLAGS + extra
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources()))
    if verbose or ptxas_info:
        for _, err in results:
            if err.strip():
                print(err, file=sys.stderr)
    tmp = LIB + ".tmp"
    cmd = [cc, "-shared", "-o", tmp] + [o for o, _ in results] + ARCH + ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv))
