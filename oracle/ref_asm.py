"""Builds oracle/_ref/libsdasm_ref.so from the reference's own x86-64 kernels -- TEST INFRASTRUCTURE ONLY.

    python oracle/ref_asm.py [--reference DIR]

DIR defaults to reference_dir(): $SDB_REFERENCE_DIR, else a directory named
"reference" beside this repository's root, where the reference's sources are.

The reference (stable-diffusion.assembly) cannot be built here as a whole: it
needs Clang >= 23, C++26 and the ggml / stable-diffusion.cpp sources, which
are absent.  Its hand-written micro-kernels are plain x86-64 assembly
(sources/x86_64/*.S), and GNU as assembles them once their C99 hex-float
literals (".float 0x1.8p23") are written as the IEEE bit patterns they denote
(".long 0x4b400000") -- the one change this recipe makes, to a build copy in
oracle/_ref/ (git-ignored; the reference's sources are not copied into the
repository).  They are linked with ref_driver.c, this project's own C code
that packs operands as the reference's gemm.cc does and calls the kernels:
    sdasm_gemm_6x16_avx2      (gemm_avx2.S)        the 6 x 16 FP32 tile
    sdasm_gated_gelu_avx2     (activation_avx2.S)  out = x GELU(gate)
    sdasm_exponentials_avx2   (softmax_avx2.S)     exp(s - max) and its sums
    sdasm_qgemm_6x16_au_avx512 (quant_avx512.S)    the quantized 6 x 16 tile (AVX512-VNNI)
    sdasm_quantize16_avx2     (quantize_avx2.S)    a panel of 16 columns quantized
The library pins the oracle (tests/test_golden.py), generates the golden
fixtures (tests/golden/make_golden.py) and, driven on all host threads
(refk_mul_mat_mt, refk_conv2d_mt), is the CPU baseline of bench.py for the
linear layers and convolutions; nothing in the product links it.
"""
from __future__ import annotations

import argparse
import os
import re
import struct
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def reference_dir() -> Path:
    """Where the reference's sources are: $SDB_REFERENCE_DIR, else ../reference
    beside the repository's root.  The directory may not exist (a GPU box gets
    only the repository and the libraries built from it)."""
    env = os.environ.get("SDB_REFERENCE_DIR")
    return Path(env) if env else HERE.parent.parent / "reference"


def reference_kernels_present() -> bool:
    return (reference_dir() / "sources" / "x86_64").is_dir()


KERNELS = ["gemm_avx2", "gemm_avx512", "activation_avx2", "softmax_avx2", "quant_avx512", "quantize_avx2"]
HEXFLOAT = re.compile(r"(?<![\w.])(-?0x[0-9a-fA-F]+(?:\.[0-9a-fA-F]*)?p[+-]?\d+)")


def _bits(token: str) -> str:
    return "0x%08x" % struct.unpack("<I", struct.pack("<f", float.fromhex(token)))[0]


def rewrite(src: str) -> str:
    """.float lines with hex-float literals become .long lines of their bit
    patterns; the // comments, which the C preprocessor strips for Clang, are
    dropped (GNU as does not read them as comments)."""
    out = []
    for line in src.splitlines():
        code = line.partition("//")[0]
        if ".float" in code and HEXFLOAT.search(code):
            head, _, values = code.partition(".float")
            items = [v.strip() for v in values.split(",") if v.strip()]
            conv = [_bits(v) if HEXFLOAT.fullmatch(v) else _bits(float(v).hex()) for v in items]
            code = head + ".long " + ", ".join(conv)
        out.append(code.rstrip())
    return "\n".join(out) + "\n"


def build(reference: Path | None = None) -> Path:
    reference = reference_dir() if reference is None else reference
    src_dir = reference / "sources" / "x86_64"
    if not src_dir.is_dir():
        raise FileNotFoundError(f"{src_dir}: the reference is not here")
    OUT.mkdir(exist_ok=True)
    objs = []
    for name in KERNELS:
        s = OUT / f"{name}.s"
        s.write_text(rewrite((src_dir / f"{name}.S").read_text()))
        o = OUT / f"{name}.o"
        subprocess.run(["as", "--64", "-o", str(o), str(s)], check=True, capture_output=True)
        objs.append(str(o))
    lib = OUT / "libsdasm_ref.so"
    subprocess.run(["gcc", "-O3", "-fopenmp", "-shared", "-fPIC", "-mavx2", "-mfma", "-mf16c", "-o", str(lib),
                    str(HERE / "ref_driver.c"), *objs, "-lm", "-Wl,-z,noexecstack"], check=True, capture_output=True)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(reference_dir()))
    print(build(Path(ap.parse_args().reference)))
    sys.exit(0)
