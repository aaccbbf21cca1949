#!/usr/bin/env python
"""Place the unmodified reference checkout under ``baseline/_ref/`` and build
its native Stage1 kernels for sm_100a, so that ``bench.py`` can time the
reference's own kernels on the same B200 as this library's.

``baseline/_ref/`` is git-ignored (the reference is not part of this
repository's source) but travels with the working tree to the GPU box.

Steps:

1. The offline install the benchmark contract names,
   ``pip install --no-index --no-build-isolation --find-links <wheelhouse>
   --target baseline/_ref <checkout>``.  The reference has neither a
   ``setup.py`` nor a ``pyproject.toml``, so this fails; its outcome is
   recorded in ``baseline/_ref/INSTALL.txt``.
2. The checkout's source directories (``baseline/``, ``reference/``,
   ``cuda/``, ``benchmarks/``, ``validation/``, ``tools/``, ``vllm/``) and its
   top-level text files are copied unchanged to
   ``baseline/_ref/turboquant-cuda-decode/``.  The profiler reports under
   ``results/`` are not copied.  The reference's harness modules
   (``baseline/triton_v1.py``, ``baseline/triton_v2.py``) load its Triton
   kernels from that copy with their own vLLM import stubs.
3. CUDA V9 (``cuda/tq4_cuda_v9.cu`` + ``cuda/tq4_cuda_v9_bind.cpp``, the
   reference's best native Stage1) and CUDA V7 (``cuda/tq4_cuda_v7.cu`` +
   ``cuda/tq4_cuda_v7_bind.cpp``: Stage1, Stage2 and the full decode) are
   compiled from the copied sources with ``torch.utils.cpp_extension`` and
   the reference's own nvcc flags (``-O3 -lineinfo --use_fast_math``,
   ``benchmarks/stage1.py:62-78``), but for ``sm_100a`` instead of the
   reference's ``sm_89``.  The extensions land in ``baseline/_ref/build_v9/``
   and ``baseline/_ref/build_v7/``; a failed build is recorded in
   ``INSTALL.txt`` with the compiler's message.

Usage::

    python baseline/install_ref.py --src <reference checkout> [--force]
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_ROOT = HERE / "_ref"
CHECKOUT = REF_ROOT / "turboquant-cuda-decode"
COPY_DIRS = ["baseline", "reference", "cuda", "benchmarks", "validation", "tools", "vllm"]
COPY_FILES = ["README.md", "THIRD_PARTY_NOTICES.md", "requirements.txt", "run.sh"]
NATIVE = {
    # name: (module name, sources relative to the checkout, build folder)
    "v9": ("tq4_cuda_v9_ext", ["cuda/tq4_cuda_v9_bind.cpp", "cuda/tq4_cuda_v9.cu"], "build_v9"),
    "v7": ("tq4_cuda_v7_ext", ["cuda/tq4_cuda_v7_bind.cpp", "cuda/tq4_cuda_v7.cu"], "build_v7"),
}
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def try_pip(src: Path) -> dict:
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--find-links", "/opt/wheelhouse", "--target", str(REF_ROOT / "pip_target"), str(src)]
    t0 = time.time()
    res = subprocess.run(cmd, capture_output=True, text=True)
    tail = (res.stdout + res.stderr).strip().splitlines()[-3:]
    return {"cmd": " ".join(cmd), "rc": res.returncode, "seconds": round(time.time() - t0, 1),
            "tail": tail}


def copy_checkout(src: Path) -> dict:
    if CHECKOUT.exists():
        shutil.rmtree(CHECKOUT)
    CHECKOUT.mkdir(parents=True)
    copied = []
    for d in COPY_DIRS:
        if (src / d).is_dir():
            shutil.copytree(src / d, CHECKOUT / d, ignore=shutil.ignore_patterns("__pycache__", "build*"))
            copied.append(d + "/")
    for f in COPY_FILES:
        if (src / f).is_file():
            shutil.copy2(src / f, CHECKOUT / f)
            copied.append(f)
    for p in CHECKOUT.rglob("*"):  # the checkout is read-only; the copy need not be
        p.chmod(p.stat().st_mode | 0o200)
    CHECKOUT.chmod(CHECKOUT.stat().st_mode | 0o200)
    return {"copied": copied}


def build_native(name: str) -> dict:
    mod, sources, folder = NATIVE[name]
    build_dir = REF_ROOT / folder
    build_dir.mkdir(parents=True, exist_ok=True)
    # torch adds -gencode flags for every entry of this list; name only the
    # B200 so the one architecture built is sm_100a (from ARCH below).
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ["PATH"] = f"{Path(sys.executable).parent}:{os.environ.get('PATH', '')}"
    from torch.utils.cpp_extension import load

    t0 = time.time()
    try:
        load(name=mod, sources=[str(CHECKOUT / s) for s in sources], extra_cflags=["-O3"],
             extra_cuda_cflags=["-O3", "-lineinfo", "--use_fast_math", *ARCH], build_directory=str(build_dir),
             with_cuda=True, verbose=False)
    except Exception as e:  # the compiler's message is the record
        return {"ok": False, "error": str(e).strip().splitlines()[-20:], "seconds": round(time.time() - t0, 1)}
    so = sorted(build_dir.glob(f"{mod}*.so"))
    return {"ok": bool(so), "so": [str(p.relative_to(HERE.parent)) for p in so],
            "flags": ["-O3", "-lineinfo", "--use_fast_math", *ARCH], "seconds": round(time.time() - t0, 1)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--src", required=True, help="the reference checkout (zben777/turboquant-cuda-decode)")
    ap.add_argument("--force", action="store_true", help="redo the copy and the native builds")
    args = ap.parse_args()
    src = Path(args.src).resolve()
    if not (src / "baseline" / "triton_v1.py").is_file():
        raise SystemExit(f"{src} is not a turboquant-cuda-decode checkout (no baseline/triton_v1.py)")
    REF_ROOT.mkdir(exist_ok=True)
    record = {"when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}
    record["pip"] = try_pip(src)
    if args.force or not (CHECKOUT / "baseline" / "triton_v1.py").is_file():
        record["copy"] = copy_checkout(src)
    else:
        record["copy"] = {"kept": str(CHECKOUT.relative_to(HERE.parent))}
    for name in NATIVE:
        record[f"cuda_{name}"] = build_native(name)
    (REF_ROOT / "INSTALL.txt").write_text(json.dumps(record, indent=1) + "\n")
    print(json.dumps(record, indent=1))


if __name__ == "__main__":
    main()
