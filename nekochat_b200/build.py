"""Builds nekochat_b200/libneko_cuda.so: every .cu under csrc/ compiled with nvcc for sm_100a only.

Used by __graft_entry__.build() and by the package on import when the library is missing in a source tree
(never on the GPU box, which receives the built library). Objects go to nekochat_b200/_build/.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libneko_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC,-O3",
                 "-I" + os.path.join(HERE, "..", "include")]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))] + [
        os.path.join(HERE, "..", "include", "neko_cuda.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = headers()
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if _stale(obj, [src] + hdrs) or ptxas_info:
            cmd = [cc] + CFLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", src, "-o", obj]
            jobs.append((src, obj, cmd))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in sources()]

    def run(job):
        src, obj, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        for src, r in ex.map(run, jobs):
            if verbose or ptxas_info:
                sys.stderr.write(r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if jobs or _stale(LIB, objs):
        cmd = [cc] + ARCH + ["-shared", "-rdc=true", "-o", LIB] + objs + [
            "-Xlinker", "--exclude-libs,ALL"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="-v" in sys.argv))
