"""Build libanimaxs_attn.so in-tree with nvcc for sm_100a (no JIT, no torch extension).

Usage: ``python -m animaxs_b200.build`` (also run by ``__graft_entry__.build()``).
Objects go to ``animaxs_b200/_build/``; the shared library to
``animaxs_b200/libanimaxs_attn.so`` so that it travels with the source tree.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libanimaxs_attn.so")
CALL_BENCH = os.path.join(BUILD, "call_bench")
SOURCES = ["attn_api.cu", "attn_fwd_sm100.cu", "attn_s3_sm100.cu", "attn_wide_sm100.cu", "qk_norm.cu", "sharded.cu",
           "noalloc.cu", "proj_api.cu", "proj_sm100.cu", "dequant_sm100.cu",
           "peer_sync.cu", "peer_sharded.cu", "cross_kv_cache.cu", "weight_streamer.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall",
         "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _headers():
    inc = os.path.join(os.path.dirname(HERE), "include")
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return hs


# Kernels that re-split their registers with setmaxnreg: source file ->
# (kernel-name pattern in the ptxas report, raised-count define, lowered-count
# define, raised-thread-count constant).
REGISTER_SPLITS = {
    "attn_fwd_sm100.cu": ("attn_fwd_sm100_kernel", "AX_SOFTMAX_REGS", "AX_OTHER_REGS", "kSoftmaxThreads"),
    "proj_sm100.cu": ("proj_sm100_kernel", "AX_EPI_REGS", "AX_PROJ_OTHER_REGS", "kEpiThreads"),
}


def check_register_split(source: str, ptxas_log: str) -> None:
    """A kernel that re-splits its registers with setmaxnreg raises some
    warpgroups' counts; the raise waits until enough registers are free in the
    CTA's launch allocation, so the new shares must fit into (threads x
    registers ptxas gave each thread at launch).  Refuse to build otherwise."""
    import re
    kernel, hi_def, lo_def, hi_threads = REGISTER_SPLITS[os.path.basename(source)]
    text = open(source).read()
    soft = int(re.search(rf"#define {hi_def} (\d+)", text).group(1))
    other = int(re.search(rf"#define {lo_def} (\d+)", text).group(1))
    threads = int(re.search(r"constexpr int kThreads = (\d+);", text).group(1))
    ms = re.search(rf"constexpr int {hi_threads} = (\d+);", text)
    softmax_threads = int(ms.group(1)) if ms else 256
    counts = re.findall(rf"entry function '[^']*{kernel}[^']*'.*?Used (\d+) registers", ptxas_log, re.S)
    if not counts:
        raise RuntimeError(f"could not read {kernel}'s register count from ptxas")
    need = softmax_threads * soft + (threads - softmax_threads) * other
    for launch in map(int, counts):  # one per template instantiation
        if need > threads * launch or soft % 8 or other % 8:
            raise RuntimeError(f"{kernel}: register split {softmax_threads}x{soft} + "
                               f"{threads - softmax_threads}x{other} = {need} exceeds the launch "
                               f"allocation {threads}x{launch} = {threads * launch}")


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    headers = _headers()
    objs, jobs = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if force or not _newer(obj, [path] + headers):
            jobs.append([cc, *ARCH, *FLAGS, "-c", path, "-o", obj])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            logs.append((cmd, res))
            if res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    if verbose:
        for cmd, res in logs:
            sys.stderr.write(f"--- {os.path.basename(cmd[-3])}\n{res.stderr}")
    for cmd, res in logs:
        if os.path.basename(cmd[-3]) in REGISTER_SPLITS:
            check_register_split(cmd[-3], res.stderr)
    if force or jobs or not _newer(LIB, objs):
        link = [cc, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-ldl", "-Xcompiler", "-fPIC"]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
        os.replace(LIB + ".tmp", LIB)
    # The C-ABI call-cost harness bench.py runs (csrc/call_bench.cu), linked
    # against the library beside this file.
    src = os.path.join(CSRC, "call_bench.cu")
    if force or not _newer(CALL_BENCH, [src, LIB] + headers):
        cmd = [cc, *ARCH, "-O2", "-std=c++17", "-o", CALL_BENCH + ".tmp", src, "-L" + HERE, "-lanimaxs_attn",
               "-Xlinker", "-rpath=$ORIGIN/.."]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("call_bench build failed")
        os.replace(CALL_BENCH + ".tmp", CALL_BENCH)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
