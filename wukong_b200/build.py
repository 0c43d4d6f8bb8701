"""Build the sm_100a op library.

Outputs (in-tree, git-ignored, shipped with the source snapshot):
  wukong_b200/libwukong.so   shared library for Python/ctypes and C hosts
  build/libwukong.a          static archive for the reference's unchanged cgo
                             line (llm/array.go:4 links ./build/libwukong.a
                             -lcublasLt -lcudart -lm -lcublas)

  wukong_b200/libwukong_timeline.so   with --timeline: the same library built
                             with -DWK_TIMELINE (per-launch decode timeline,
                             python -m wukong_b200.timeline)

Usage: python -m wukong_b200.build [-j N] [--force] [--timeline]
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
SO = os.path.join(HERE, "libwukong.so")
TIMELINE_SO = os.path.join(HERE, "libwukong_timeline.so")
ARCHIVE = os.path.join(ROOT, "build", "libwukong.a")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fno-exceptions", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(src, obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + deps)


def _compile(src, obj, extra):
    cmd = [NVCC] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(jobs=8, force=False, verbose=False, ptxas_v=False, timeline=False):
    obj_dir = OBJ + "_timeline" if timeline else OBJ
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(os.path.dirname(ARCHIVE), exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _headers()
    extra = (["-Xptxas", "-v"] if ptxas_v else []) + (["-DWK_TIMELINE"] if timeline else [])
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(obj_dir, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or ptxas_v or _stale(s, o, deps):
            todo.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = {ex.submit(_compile, s, o, extra): s for s, o in todo}
        for f in cf.as_completed(futs):
            msg = f.result()
            if verbose and msg:
                print(f"== {os.path.basename(futs[f])}\n{msg}")
    if timeline:
        if todo or not os.path.exists(TIMELINE_SO):
            subprocess.check_call([NVCC] + ARCH + ["-shared", "-o", TIMELINE_SO] + objs + ["-ldl"])
        return TIMELINE_SO
    if todo or not os.path.exists(SO) or not os.path.exists(ARCHIVE):
        subprocess.check_call([NVCC] + ARCH + ["-shared", "-o", SO] + objs + ["-ldl"])
        if os.path.exists(ARCHIVE):
            os.remove(ARCHIVE)
        subprocess.check_call([NVCC] + ARCH + ["-lib", "-o", ARCHIVE] + objs)
    return SO


def main():
    p = argparse.ArgumentParser()
    p.add_argument("-j", type=int, default=8)
    p.add_argument("--force", action="store_true")
    p.add_argument("--ptxas-v", action="store_true", help="print registers / spills / shared memory per kernel")
    p.add_argument("--timeline", action="store_true", help="build libwukong_timeline.so (-DWK_TIMELINE)")
    a = p.parse_args()
    print(build(a.j, a.force, verbose=True, ptxas_v=a.ptxas_v, timeline=a.timeline))


if __name__ == "__main__":
    sys.exit(main())
