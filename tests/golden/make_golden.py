#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory.

Block-scheme goldens come from the reference's own generator,
``tests/gen_reference.py`` of nim-lowprec, imported from the reference checkout
with its output directory redirected here (the checkout is read-only):

  * ``emit_ggml_schemes`` (gen_reference.py:151-196): seed 1234, n = 16384,
    x = N(0,1)*4 with an all-zero block and a 1e-30 block; Q8_0/Q4_0 quantize
    bytes and their dequant from gguf-py (llama.cpp's numpy implementation).
  * ``emit_mx_schemes`` (gen_reference.py:199-234): seed 777, 512 blocks with a
    2^-140..2^120 magnitude sweep; OCP-MX fp4 calibrate+quantize+dequant with
    ml_dtypes element rounding.

Element-codec goldens (e2m1, E8M0, f16) follow the same recipe as
gen_reference.py's ``emit_mx_float``/``emit_e8m0``/``emit_f16`` (edges plus a
seeded random sample, answers from ml_dtypes / numpy) but with a smaller random
sample so the fixtures stay a few hundred KB.

Run from anywhere:  python tests/golden/make_golden.py [path/to/reference]
Only this script needs the reference checkout; the tests read the fixtures.
"""
import importlib.util
import os
import sys

import ml_dtypes
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_generator(ref_root):
    path = os.path.join(ref_root, "tests", "gen_reference.py")
    spec = importlib.util.spec_from_file_location("gen_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.HERE = HERE  # write into this directory, never into the checkout
    return mod


def element_codecs():
    # e2m1 encode: finite edges + random sample (gen_reference.py:95-118 recipe)
    edge_vals = np.array([0.0, -0.0, 0.25, 0.5, 1.0, -1.0, 1.5, -1.5, 2.0, 3.0, 4.0, 6.0, 7.0,
                          7.5, 8.0, 28.0, 100.0, -100.0, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                          -0.25, -0.75, -2.5, -5.0, np.inf, -np.inf], dtype=np.float32)
    rng = np.random.default_rng(41)
    rand = rng.integers(0, 1 << 32, size=60_000, dtype=np.uint64).astype(np.uint32)
    # plus values inside the e2m1 range, where the rounding decisions are
    near = (rng.standard_normal(20_000) * 3.0).astype(np.float32).view(np.uint32)
    ins = np.unique(np.concatenate([edge_vals.view(np.uint32), rand, near])).astype(np.uint32)
    f = ins.view(np.float32)
    ins = ins[~np.isnan(f)]  # NaN inputs are undefined for a finite format
    with np.errstate(over="ignore", invalid="ignore"):
        outs = ins.view(np.float32).astype(ml_dtypes.float4_e2m1fn).view(np.uint8)
    np.savez_compressed(os.path.join(HERE, "e2m1_encode.npz"), ins=ins, outs=outs)

    # E8M0 encode, normal positive inputs (gen_reference.py:121-143 recipe)
    edge = np.array([1.0, 1.4, 1.5, 1.9, 2.0, 2.9, 3.0, 0.4, 0.75, 6.0, 2.0 ** -126, 2.0 ** 126,
                     2.0 ** 127, 0.0, np.inf, np.nan], dtype=np.float32)
    rng = np.random.default_rng(23)
    rand = rng.integers(0x00800000, 0x7f800000, size=60_000, dtype=np.uint64).astype(np.uint32)
    ins = np.unique(np.concatenate([edge.view(np.uint32), rand])).astype(np.uint32)
    with np.errstate(over="ignore", invalid="ignore"):
        outs = ins.view(np.float32).astype(ml_dtypes.float8_e8m0fnu).view(np.uint8)
    np.savez_compressed(os.path.join(HERE, "e8m0_encode.npz"), ins=ins, outs=outs)

    # f32 -> f16 (gen_reference.py:47-74 recipe)
    edges = np.array([0x00000000, 0x80000000, 0x3F800000, 0xBF800000, 0x7F800000, 0xFF800000,
                      0x7F800001, 0x7FC00000, 0x477FE000, 0x47800000, 0x38800000, 0x33800000,
                      0x33000000, 0x38000000], dtype=np.uint32)
    rng = np.random.default_rng(1)
    rand = rng.integers(0, 1 << 32, size=100_000, dtype=np.uint64).astype(np.uint32)
    ins = np.unique(np.concatenate([edges, rand])).astype(np.uint32)
    with np.errstate(over="ignore", invalid="ignore"):
        outs = ins.view(np.float32).astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "f16_encode.npz"), ins=ins, outs=outs)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NIM_LOWPREC_REF")
    if not ref_root:
        sys.exit("usage: make_golden.py <nim-lowprec checkout> (or set NIM_LOWPREC_REF)")
    gen = load_reference_generator(ref_root)
    gen.emit_ggml_schemes()
    gen.emit_mx_schemes()
    gen.emit_nvfp4()
    # keep only the fixtures this repository tests against
    for name in ("ref_mx_f6e2m3_dq.bin", "ref_mx_f6e3m2_dq.bin"):
        p = os.path.join(HERE, name)
        if os.path.exists(p):
            os.remove(p)
    element_codecs()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
