"""Build libq3attn.so in-tree for sm_100a (B200) with nvcc.

    python -m q3attn.build            (from qwen3-tts-engine_b200/)   or   q3attn.build.build()

Every .cu under qwen3-tts-engine_b200/csrc is compiled separately (in parallel) and linked into
qwen3-tts-engine_b200/q3attn/libq3attn.so next to this file, where q3attn._lib loads it. Objects go to
qwen3-tts-engine_b200/_build/. The library is rebuilt unless the SHA-256 of every source, header and this script (and
the nvcc flags) equals the digest stamped beside it when it was last built, so a copied tree never runs a library that
was built from other sources, whatever the files' modification times say.
"""
import concurrent.futures as cf
import glob
import hashlib
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
STAMP = LIB + ".sha256"
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


def source_digest() -> str:
    """SHA-256 over the build inputs: each dependency's name and bytes, in name order, plus the nvcc flags."""
    h = hashlib.sha256(" ".join(NVCC_FLAGS).encode())
    for d in sorted(set(_deps())):
        h.update(os.path.basename(d).encode() + b"\0")
        with open(d, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def up_to_date() -> bool:
    if not (os.path.exists(LIB) and os.path.exists(STAMP)):
        return False
    with open(STAMP) as f:
        return f.read().strip() == source_digest()


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
    with open(STAMP, "w") as f:
        f.write(source_digest() + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv))
