"""Build the sm_100a kernel library in-tree and write its manifest.

Output: ``h3_speedkit/_native/libh3sk_b200.so`` plus one symlink per library
name the reference loads (``norm.so``, ``residual.so``, ``convrot.so``, ``fc1.so``, ``gate.so``, ``qkv.so``,
``sample.so``, ``anchor.so``)
and ``build.json`` in the reference's manifest schema
(tools/build_kernels.py:41-63 of H3 SpeedKit: schema, kernels[name].sha256 ...).

The quantiser translation units are compiled with ``--use_fast_math`` exactly
as the reference compiles its norm/convrot kernels (tools/build_kernels.py:32-34),
because the quantiser's division must be the same operation; the GEMM unit is
compiled without it and spells every epilogue rounding explicitly.  The QKV head
epilogue is compiled without it and the K anchor detector and the INT8
attention with it, as the reference compiles its qkv/sample, anchor and dense
units (tools/build_kernels.py:30-37).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
NATIVE = PKG / "h3_speedkit" / "_native"
BUILD = PKG / "_build"
LIB_NAME = "libh3sk_b200.so"
ALIASES = ("norm", "residual", "convrot", "fc1", "gate", "qkv", "sample", "anchor", "dense")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-DNDEBUG", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
          "--expt-relaxed-constexpr"]
UNITS = (
    ("norm_quant.cu", ["--use_fast_math", "-DH3SK_QUANT_FAST_MATH"]),
    ("convrot_quant.cu", ["--use_fast_math", "-DH3SK_QUANT_FAST_MATH"]),
    ("int8_gemm.cu", []),
    ("qkv_quant.cu", []),
    ("anchor.cu", ["--use_fast_math"]),
    ("attention.cu", ["--use_fast_math"]),
)


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def nvcc_path(explicit: str | None = None) -> str:
    for candidate in (explicit, shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the sm_100a library")


def up_to_date() -> bool:
    lib = NATIVE / LIB_NAME
    if not lib.exists() or not (NATIVE / "build.json").exists():
        return False
    newest = max(p.stat().st_mtime for p in list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                 + [PKG.parent / "include" / "h3sk_b200.h", Path(__file__)])
    return lib.stat().st_mtime >= newest


def build(nvcc: str | None = None, force: bool = False, quiet: bool = True) -> Path:
    if not force and up_to_date():
        return NATIVE / LIB_NAME
    nvcc = nvcc_path(nvcc)
    BUILD.mkdir(parents=True, exist_ok=True)
    NATIVE.mkdir(parents=True, exist_ok=True)
    version = subprocess.check_output([nvcc, "--version"], text=True)
    manifest = {"schema": 1, "status": "building", "target": "sm_100a", "nvcc": version, "kernels": {}}
    objects, logs, commands = [], [], {}
    for source, extra in UNITS:
        src = CSRC / source
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, *COMMON, *ARCH, *extra, "-c", str(src), "-o", str(obj)]
        result = subprocess.run(cmd, text=True, capture_output=True)
        logs.append(f"$ {' '.join(cmd)}\n{result.stdout}{result.stderr}")
        commands[source] = cmd
        if result.returncode:
            (NATIVE / "build.log").write_text("\n".join(logs))
            raise RuntimeError(f"nvcc failed on {source}:\n{result.stderr[-6000:]}")
        objects.append(obj)
    lib = NATIVE / LIB_NAME
    tmp = NATIVE / (LIB_NAME + ".tmp")
    link = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp)]
    result = subprocess.run(link, text=True, capture_output=True)
    logs.append(f"$ {' '.join(link)}\n{result.stdout}{result.stderr}")
    (NATIVE / "build.log").write_text("\n".join(logs))
    if result.returncode:
        raise RuntimeError(f"link failed:\n{result.stderr[-4000:]}")
    os.replace(tmp, lib)
    digest = sha256(lib)
    sources = {"norm": "norm_quant.cu", "residual": "norm_quant.cu", "convrot": "convrot_quant.cu",
               "fc1": "int8_gemm.cu", "gate": "int8_gemm.cu", "qkv": "qkv_quant.cu", "sample": "qkv_quant.cu",
               "anchor": "anchor.cu", "dense": "attention.cu"}
    for name in ALIASES:
        alias = NATIVE / (name + ".so")
        if alias.is_symlink() or alias.exists():
            alias.unlink()
        alias.symlink_to(LIB_NAME)
        src = CSRC / sources[name]
        manifest["kernels"][name] = {"source": f"csrc/{sources[name]}", "source_sha256": sha256(src),
                                     "exit_code": 0, "command": commands[sources[name]],
                                     "library": LIB_NAME, "sha256": digest}
    manifest["status"] = "compiled; numerical validation required"
    (NATIVE / "build.json").write_text(json.dumps(manifest, indent=2) + "\n")
    if not quiet:
        print(f"built {lib} ({lib.stat().st_size} bytes)")
    return lib


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--nvcc")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    build(args.nvcc, force=args.force, quiet=False)
    return 0


if __name__ == "__main__":
    sys.exit(main())
