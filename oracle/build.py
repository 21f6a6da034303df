"""Build the oracles.  TEST INFRASTRUCTURE ONLY.

1. ``oracle/libh3_oracle.so`` -- the C restatement (h3_oracle.c), built with gcc,
   -ffp-contract=off, no fast-math, OpenMP, baseline x86-64 code (it travels to
   the GPU box, whose CPU may differ from the build host).
2. ``oracle/_ref/*.so`` -- the reference's own CUDA kernels, compiled from the
   sources where they lie under the reference checkout (never copied into this
   repository) with the reference's flags (tools/build_kernels.py:26-40) and the
   architecture switched to sm_100a:
     * ``ref_norm_k{K}.so``  kernels/norm_quant/norm_quant.cu.  The reference fixes
       ``K = 5376`` in a constexpr (norm_quant.cu:16); for other widths this
       recipe writes a derived copy with only that constant changed into
       ``oracle/_ref/gen/``, compiles it and deletes it again (only the .so stays);
     * ``ref_convrot.so``    kernels/convrot/convrot_register_v2.cu, unmodified
       (K in {5376, 7168});
     * ``ref_kitchen.so``    oracle/ref_kitchen_launch.cu, which instantiates the
       vendored Kitchen quantiser of kernels/convrot/vendor/convrot64_exact.cuh.
     * ``ref_residual_k{K}.so`` kernels/residual_quant/residual_quant.cu (the
       reference's residual update fused with the prologue; K fixed the same way
       as norm_quant.cu, rewritten the same way for K = 4096);
     * ``ref_anchor.so``     kernels/gemm/r79_sample_anchor.cu, unmodified (the K
       anchor detector ``h3_sample_anchor``; plain CUDA, --use_fast_math);
     * ``ref_gather.so``     kernels/gemm/r82_sample_konly.cu, unmodified, built
       without ``COMFY_HAVE_CUTLASS``: that leaves exactly its sample-row gather
       ``h3_sample_gather`` (the CUTLASS K-only GEMM is compiled out);
     * ``ref_fc1.so``        kernels/gemm/fc1.cu, unmodified (``h3_int8``, the
       CUTLASS 2.x Sm80 INT8 GEMM with the dequant EVT epilogue), flags
       ``-DCOMFY_HAVE_CUTLASS -DH3_EVT_STAGES=2``;
     * ``ref_gate.so``       kernels/gemm/gate.cu, unmodified (``h3_int8_gate``,
       the gate-residual EVT epilogue, configs 0 and 13), ``-DH3_EVT_STAGES=1``;
     * ``ref_dense.so``      kernels/dense/dense_ring.cu, unmodified (the INT8
       attention ``h3_dense_launch_window``, variant 8102), with the reference's
       dense flags (``--use_fast_math -lineinfo --maxrregcount=168
       -DH3_VARIANT_ID=8102 -lcuda``) and ``sm_100a`` in place of ``sm_120a``;
     * ``ref_qkv.so``        kernels/gemm/r84_kfourwarp.cu, unmodified
       (``h3_qkv_quant_kv``, the QKV GEMM fused with the per-head RMS / RoPE /
       rotation / quantisation epilogue), ``-DH3_EVT_STAGES=2``.
   The three GEMM units need CUTLASS headers.  The reference pins CUTLASS 4.5.0
   (configs/compatibility.json:19); the recipe takes them from ``H3SK_CUTLASS``
   (a directory holding ``cutlass/cutlass.h``) or else from the copy that the
   flashinfer wheel ships (``flashinfer/data/cutlass/include``, also 4.5.0), and
   skips those three libraries with a notice when neither exists.
   Step 2 runs only where the reference checkout exists (the build host); the
   GPU box uses the prebuilt files.  The checkout is ``H3SK_REFERENCE`` or, when
   that is unset, a directory named ``reference`` beside this repository.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
REFERENCE = Path(os.environ.get("H3SK_REFERENCE") or HERE.parent.parent / "reference")
C_LIB = HERE / "libh3_oracle.so"
NORM_WIDTHS = (2048, 4096, 5376)
RESIDUAL_WIDTHS = (4096, 5376)
REF_FLAGS = ["-std=c++20", "-O3", "-DNDEBUG", "--expt-relaxed-constexpr", "--expt-extended-lambda",
             "--shared", "-Xcompiler=-fPIC", "-gencode=arch=compute_100a,code=sm_100a"]


def _newer(target: Path, *sources: Path) -> bool:
    return target.exists() and all(target.stat().st_mtime >= s.stat().st_mtime for s in sources if s.exists())


def build_c(force: bool = False) -> Path:
    src = HERE / "h3_oracle.c"
    if not force and _newer(C_LIB, src, Path(__file__)):
        return C_LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the CPU oracle")
    tmp = C_LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-std=c11", "-fno-fast-math", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
           "-fvisibility=hidden", str(src), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, C_LIB)
    return C_LIB


def _nvcc() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc is required to build the reference GPU oracle")


def _compile(nvcc: str, source: Path, target: Path, includes: list[Path], extra: list[str]) -> None:
    cmd = [nvcc, *REF_FLAGS, *extra, *(f"-I{p}" for p in includes), str(source), "-o", str(target)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"reference oracle build failed for {source.name}:\n{result.stderr[-4000:]}")


def build_ref(force: bool = False) -> list[Path]:
    """Compile the reference kernels into oracle/_ref (needs the reference checkout)."""
    kernels = REFERENCE / "kernels"
    if not (kernels / "norm_quant" / "norm_quant.cu").exists():
        return sorted(REF_OUT.glob("*.so"))
    nvcc = _nvcc()
    REF_OUT.mkdir(exist_ok=True)
    gen = REF_OUT / "gen"
    gen.mkdir(exist_ok=True)
    built = []
    norm_src = kernels / "norm_quant" / "norm_quant.cu"
    text = norm_src.read_text()
    pattern = re.compile(r"constexpr int K = 5376,")
    if len(pattern.findall(text)) != 1:
        raise RuntimeError("norm_quant.cu no longer has the single K constant this recipe rewrites")
    for k in NORM_WIDTHS:
        target = REF_OUT / f"ref_norm_k{k}.so"
        if force or not _newer(target, norm_src, Path(__file__)):
            source = norm_src if k == 5376 else gen / f"norm_quant_k{k}.cu"
            if k != 5376:
                source.write_text(pattern.sub(f"constexpr int K = {k},", text))
            try:
                _compile(nvcc, source, target, [norm_src.parent, norm_src.parent / "vendor"],
                         ["--use_fast_math"])
            finally:
                if k != 5376:
                    source.unlink(missing_ok=True)
        built.append(target)
    res_src = kernels / "residual_quant" / "residual_quant.cu"
    res_text = res_src.read_text()
    if len(pattern.findall(res_text)) != 1:
        raise RuntimeError("residual_quant.cu no longer has the single K constant this recipe rewrites")
    for k in RESIDUAL_WIDTHS:
        target = REF_OUT / f"ref_residual_k{k}.so"
        if force or not _newer(target, res_src, Path(__file__)):
            source = res_src if k == 5376 else gen / f"residual_quant_k{k}.cu"
            if k != 5376:
                source.write_text(pattern.sub(f"constexpr int K = {k},", res_text))
            try:
                _compile(nvcc, source, target, [res_src.parent, res_src.parent / "vendor"], ["--use_fast_math"])
            finally:
                if k != 5376:
                    source.unlink(missing_ok=True)
        built.append(target)
    conv_src = kernels / "convrot" / "convrot_register_v2.cu"
    target = REF_OUT / "ref_convrot.so"
    if force or not _newer(target, conv_src):
        _compile(nvcc, conv_src, target, [conv_src.parent, conv_src.parent / "vendor"], ["--use_fast_math"])
    built.append(target)
    gemm_dir = kernels / "gemm"
    for name, source, extra in (("ref_anchor.so", "r79_sample_anchor.cu", ["--use_fast_math"]),
                                ("ref_gather.so", "r82_sample_konly.cu", [])):
        target = REF_OUT / name
        if force or not _newer(target, gemm_dir / source):
            _compile(nvcc, gemm_dir / source, target, [gemm_dir], extra)
        built.append(target)
    launcher = HERE / "ref_kitchen_launch.cu"
    target = REF_OUT / "ref_kitchen.so"
    vendor = kernels / "convrot" / "vendor"
    if force or not _newer(target, launcher, vendor / "convrot64_exact.cuh"):
        _compile(nvcc, launcher, target, [vendor], ["--use_fast_math"])
    built.append(target)
    built += _build_ref_gemms(nvcc, gemm_dir, force)
    dense_dir = kernels / "dense"
    target = REF_OUT / "ref_dense.so"
    if force or not _newer(target, *sorted(dense_dir.glob("*"))):
        _compile(nvcc, dense_dir / "dense_ring.cu", target, [dense_dir],
                 ["--use_fast_math", "-lineinfo", "--maxrregcount=168", "-DH3_VARIANT_ID=8102", "-lcuda"])
    built.append(target)
    return built


# (library, source in kernels/gemm, the reference's flags for it: tools/build_kernels.py:35-39)
REF_GEMMS = (("ref_fc1.so", "fc1.cu", ["-DCOMFY_HAVE_CUTLASS", "-DH3_EVT_STAGES=2"]),
             ("ref_gate.so", "gate.cu", ["-DCOMFY_HAVE_CUTLASS", "-DH3_EVT_STAGES=1"]),
             ("ref_qkv.so", "r84_kfourwarp.cu", ["-DCOMFY_HAVE_CUTLASS", "-DH3_EVT_STAGES=2"]))


def cutlass_include() -> Path | None:
    """CUTLASS headers for the reference GEMM units: ``H3SK_CUTLASS`` or flashinfer's copy."""
    env = os.environ.get("H3SK_CUTLASS")
    candidates = [Path(env)] if env else []
    try:
        import importlib.util
        spec = importlib.util.find_spec("flashinfer")
        if spec and spec.submodule_search_locations:
            candidates += [Path(p) / "data" / "cutlass" / "include" for p in spec.submodule_search_locations]
    except (ImportError, ValueError):
        pass
    for c in candidates:
        if (c / "cutlass" / "cutlass.h").is_file():
            return c
    return None


def _build_ref_gemms(nvcc: str, gemm_dir: Path, force: bool) -> list[Path]:
    """Compile fc1.cu, gate.cu and r84_kfourwarp.cu in parallel (each takes about a minute)."""
    todo = [(REF_OUT / name, gemm_dir / src, extra) for name, src, extra in REF_GEMMS
            if force or not _newer(REF_OUT / name, gemm_dir / src, gemm_dir / "cutlass_gemm_common.cuh")]
    done = [REF_OUT / name for name, _, _ in REF_GEMMS if (REF_OUT / name).exists()]
    if not todo:
        return done
    include = cutlass_include()
    if include is None:
        print("oracle: CUTLASS headers not found (set H3SK_CUTLASS); reference GEMM oracles not built",
              file=sys.stderr)
        return [p for p in done if p not in {t for t, _, _ in todo}]
    procs = []
    for target, source, extra in todo:
        tmp = target.with_suffix(".so.tmp")
        cmd = [nvcc, *REF_FLAGS, *extra, f"-I{include}", f"-I{gemm_dir}", str(source), "-o", str(tmp)]
        procs.append((target, tmp, source, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                                            text=True)))
    failures = []
    for target, tmp, source, proc in procs:
        _, err = proc.communicate()
        if proc.returncode:
            failures.append(f"{source.name}:\n{err[-4000:]}")
        else:
            os.replace(tmp, target)
    if failures:
        raise RuntimeError("reference GEMM oracle build failed for " + "\n".join(failures))
    return [REF_OUT / name for name, _, _ in REF_GEMMS]


def build(force: bool = False) -> None:
    build_c(force)
    build_ref(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print("oracle built:", C_LIB, *sorted(p.name for p in REF_OUT.glob("*.so")))
