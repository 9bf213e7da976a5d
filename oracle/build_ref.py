"""Build the reference's own AOT tools into oracle/_ref/ — test infrastructure.

Compiles, with g++ directly on the reference's sources where they lie:

  oracle/_ref/gawee-aot    back/gawee_aot.cpp   (launcher generator of `gawee-aot build`)
  oracle/_ref/gawee-eval   back/gawee_eval.cpp  (`gawee-eval compare|benchmark`)

and, for a few small graphs, the runner the reference's flow would produce,
with the B200 backend in place of the lowered CPU object:

  oracle/_ref/aot/<name>/forward.mlir         the gawee graph
  oracle/_ref/aot/<name>/forward_memref.mlir  its bufferized signature (gawee_b200.aot abi)
  oracle/_ref/aot/<name>/launcher.cpp         written by the reference's gawee-aot (--dump-launcher)
  oracle/_ref/aot/<name>/forward_shim.c       gawee_b200.aot shim (what --gawee-to-cuda emits)
  oracle/_ref/aot/<name>/runner               launcher + shim + back/runtime_support.h, -lgawee_cuda

The reference's `gawee-aot build` stops after dumping the launcher, at its
`llc` step (back/gawee_aot.cpp:331-340): there is no LLVM toolchain here, and
the lowered object is replaced by the shim anyway.  Everything is written
under oracle/_ref/ (git-ignored; it travels with the tree to GPU machines,
where the GPU tests run the runners and compare with `gawee-eval compare`).

    python oracle/build_ref.py [--reference DIR]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
DEFAULT_REF = "/root/reference"

# name -> synth builder call; kept small so the GPU tests run them in seconds
GRAPHS = {
    "resnet18_b1_64": ("resnet18", dict(batch=1, image=64)),
    "bert_tiny_s16": ("bert_tiny", dict(seq=16, vocab=64, max_pos=32)),
}


def graph(name: str):
    sys.path.insert(0, ROOT)
    from gawee_b200 import synth
    fn, kw = GRAPHS[name]
    return getattr(synth, fn)(**kw)


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)} failed:\n{r.stdout}\n{r.stderr}")
    return r


def _newer(out: str, *srcs: str) -> bool:
    return os.path.exists(out) and all(os.path.getmtime(out) >= os.path.getmtime(s) for s in srcs)


def build(ref: str = DEFAULT_REF, force: bool = False) -> bool:
    back = os.path.join(ref, "back")
    if not os.path.isfile(os.path.join(back, "gawee_aot.cpp")):
        return False
    os.makedirs(OUT, exist_ok=True)
    hdr = os.path.join(back, "runtime_support.h")
    tools = {"gawee-aot": os.path.join(back, "gawee_aot.cpp"), "gawee-eval": os.path.join(back, "gawee_eval.cpp")}
    for name, src in tools.items():
        out = os.path.join(OUT, name)
        if force or not _newer(out, src, hdr):
            _run(["g++", "-std=c++17", "-O2", "-I" + back, src, "-o", out])

    sys.path.insert(0, ROOT)
    from gawee_b200 import aot, build as native
    lib = native.build()
    for name in GRAPHS:
        d = os.path.join(OUT, "aot", name)
        os.makedirs(d, exist_ok=True)
        text = graph(name).mlir
        paths = {k: os.path.join(d, k) for k in
                 ("forward.mlir", "forward_memref.mlir", "launcher.cpp", "forward_shim.c", "runner")}
        old = open(paths["forward.mlir"]).read() if os.path.exists(paths["forward.mlir"]) else None
        if old != text:
            with open(paths["forward.mlir"], "w") as f:
                f.write(text)
        with open(paths["forward_memref.mlir"], "w") as f:
            f.write(aot.abi_source(text))
        with open(paths["forward_shim.c"], "w") as f:
            f.write(aot.emit_ciface_shim(text))
        if not force and _newer(paths["runner"], paths["forward.mlir"], lib, hdr, os.path.join(OUT, "gawee-aot")):
            continue
        if os.path.exists(paths["launcher.cpp"]):
            os.remove(paths["launcher.cpp"])
        # the reference's generator writes the launcher, then fails at its llc step (expected)
        subprocess.run([os.path.join(OUT, "gawee-aot"), "build", "--abi-source", paths["forward_memref.mlir"],
                        "--input", os.path.join(d, "lowered.ll"), "--output", os.path.join(d, "unused"),
                        "--llvm-bin", os.path.join(d, "no-llvm"), "--dump-launcher", paths["launcher.cpp"]],
                       capture_output=True, text=True)
        if not os.path.exists(paths["launcher.cpp"]):
            raise RuntimeError(f"gawee-aot did not write the launcher for {name}")
        shim_o = os.path.join(d, "forward_shim.o")
        _run(["gcc", "-O2", "-c", paths["forward_shim.c"], "-o", shim_o])
        rel = os.path.relpath(os.path.dirname(lib), d)
        _run(["g++", "-std=c++17", "-O2", "-I" + back, paths["launcher.cpp"], shim_o, "-o", paths["runner"],
              "-L" + os.path.dirname(lib), "-lgawee_cuda", "-Wl,-rpath,$ORIGIN/" + rel])
    return True


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REF)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    ok = build(a.reference, a.force)
    print("built" if ok else f"no reference sources under {a.reference}; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
