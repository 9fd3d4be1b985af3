"""Extract the reference's double-double golden vectors into compact fixtures.

The vkfft-rs crate commits binary128 reference outputs for its DoubleDouble precisions
under ``tests/fixtures/``: ``quad_precision_medium_double_double_v1.txt`` (double-double
inputs and outputs, direct 113-bit DFT with Kahan summation rounded to hi + lo) and
``quad_precision_medium_dd_f64_storage_v1.txt`` (binary64 inputs, outputs rounded to
binary64).  The GPU box has no copy of the reference, so this script converts both into
``quad_dd_golden.npz`` next to itself.

Run once in a container that has the reference mounted::

    python tests/golden/make_dd_golden.py /path/to/vkfft-rs

Layout: for every case ``<set>/<name>`` (sets ``dd`` and ``dd_f64``) the arrays
``shape`` (int64), ``kind`` (0 = c2c, 1 = r2c, 2 = dct2), ``input`` and ``output`` as
float64 words -- ``dd``: (count, 4) per complex value (re.hi, re.lo, im.hi, im.lo) and
(count, 2) per real value (hi, lo); ``dd_f64``: (count, 2) per complex value (re, im)
and (count,) per real value.
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KINDS = {"c2c": 0, "r2c": 1, "dct2": 2}


def word(h):
    return struct.unpack("<d", struct.pack("<Q", int(h, 16)))[0]


def parse(path):
    with open(path) as fh:
        lines = [ln.rstrip("\n") for ln in fh]
    i = 0
    while not lines[i].startswith("case "):
        i += 1
    cases = {}
    while i < len(lines):
        name = lines[i][len("case "):]
        kind = lines[i + 1][len("kind "):]
        shape = [int(v) for v in lines[i + 2][len("shape "):].split()]
        n_in = int(lines[i + 4][len("input-count "):])
        n_out = int(lines[i + 6][len("output-count "):])
        i += 7
        inp = np.array([[word(h) for h in ln.split()] for ln in lines[i:i + n_in]])
        i += n_in
        assert lines[i] == "output-data", lines[i]
        i += 1
        out = np.array([[word(h) for h in ln.split()] for ln in lines[i:i + n_out]])
        i += n_out
        cases[name] = dict(kind=KINDS[kind], shape=shape, input=inp.squeeze(-1) if inp.shape[1] == 1 else inp,
                           output=out.squeeze(-1) if out.shape[1] == 1 else out)
    return cases


def main(ref_root):
    fx = os.path.join(ref_root, "tests", "fixtures")
    sets = {"dd": parse(os.path.join(fx, "quad_precision_medium_double_double_v1.txt")),
            "dd_f64": parse(os.path.join(fx, "quad_precision_medium_dd_f64_storage_v1.txt"))}
    arrays = {}
    for set_name, cases in sets.items():
        for name, case in cases.items():
            key = f"{set_name}/{name}"
            arrays[key + "/shape"] = np.array(case["shape"], dtype=np.int64)
            arrays[key + "/kind"] = np.array(case["kind"], dtype=np.int64)
            arrays[key + "/input"] = case["input"].astype(np.float64)
            arrays[key + "/output"] = case["output"].astype(np.float64)
    out = os.path.join(HERE, "quad_dd_golden.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}: {sum(len(c) for c in sets.values())} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.relpath(__file__)} <vkfft-rs checkout>")
    main(sys.argv[1])
