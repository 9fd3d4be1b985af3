"""Extract the reference's FFTW golden vectors into compact fixtures.

The vkfft-rs crate commits FFTW 3.3.9 outputs under ``tests/fixtures/`` (see
``tests/fixtures/README.md`` of the crate).  The GPU box has no copy of the
reference, so this script parses the C2C, R2C and DCT-II (FFTW REDFT10) cases and
stores them as ``fftw_golden.npz`` next to itself.

Run once in a container that has the reference mounted::

    python tests/golden/make_golden.py /path/to/vkfft-rs

Layout of the archive: for every case ``<set>/<name>`` there are arrays
``<set>/<name>/shape`` (int64), ``<set>/<name>/kind`` (0 = c2c, 1 = r2c,
2 = dct2), ``<set>/<name>/output`` (complex128; float64 for dct2) and, for the
compact set whose inputs are stored inline, ``<set>/<name>/input`` (complex128 or
float64).

Sets: ``medium`` (fftw_precision_medium_v1.txt, f64 input formulas),
``medium_f32`` (fftw_precision_medium_f32_v1.txt, inputs evaluated in float),
``compact`` (fftw_precision_v1.txt, inputs inline).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def parse_medium(path):
    cases = {}
    with open(path) as fh:
        lines = [ln.rstrip("\n") for ln in fh]
    i = 0
    while i < len(lines) and not lines[i].startswith("case "):
        i += 1
    while i < len(lines):
        name = lines[i][len("case "):]
        kind = lines[i + 1][len("kind "):]
        shape = [int(v) for v in lines[i + 2][len("shape "):].split()]
        count = int(lines[i + 4][len("output "):])
        body = lines[i + 5:i + 5 + count]
        i += 5 + count
        if kind not in ("c2c", "r2c", "dct2"):
            continue
        vals = np.array([[float(v) for v in ln.split()] for ln in body])
        out = vals[:, 0] if kind == "dct2" else vals[:, 0] + 1j * vals[:, 1]
        cases[name] = dict(kind=kind, shape=shape, output=out)
    return cases


def parse_compact(path):
    cases = {}
    with open(path) as fh:
        lines = [ln.rstrip("\n") for ln in fh]
    i = 0
    while i < len(lines) and not lines[i].startswith("case "):
        i += 1
    while i < len(lines):
        name = lines[i][len("case "):]
        kind = lines[i + 1][len("kind "):]
        n = int(lines[i + 2][len("length "):])
        i += 3
        if kind == "c2c":
            vals = np.array([[float(v) for v in ln.split()] for ln in lines[i:i + n]])
            i += n
            cases[name] = dict(kind=kind, shape=[n], input=vals[:, 0] + 1j * vals[:, 1],
                               output=vals[:, 2] + 1j * vals[:, 3])
        elif kind == "r2c":
            inp = np.array([float(ln) for ln in lines[i:i + n]])
            i += n
            count = int(lines[i][len("output "):])
            vals = np.array([[float(v) for v in ln.split()] for ln in lines[i + 1:i + 1 + count]])
            i += 1 + count
            cases[name] = dict(kind=kind, shape=[n], input=inp, output=vals[:, 0] + 1j * vals[:, 1])
        elif kind == "dct2":
            vals = np.array([[float(v) for v in ln.split()] for ln in lines[i:i + n]])
            i += n
            cases[name] = dict(kind=kind, shape=[n], input=vals[:, 0], output=vals[:, 1])
        else:
            # skip any other case kind: consume until the next "case" line
            while i < len(lines) and not lines[i].startswith("case "):
                i += 1
    return cases


def main(ref_root):
    fx = os.path.join(ref_root, "tests", "fixtures")
    sets = {
        "medium": parse_medium(os.path.join(fx, "fftw_precision_medium_v1.txt")),
        "medium_f32": parse_medium(os.path.join(fx, "fftw_precision_medium_f32_v1.txt")),
        "compact": parse_compact(os.path.join(fx, "fftw_precision_v1.txt")),
    }
    arrays = {}
    for set_name, cases in sets.items():
        for name, case in cases.items():
            key = f"{set_name}/{name}"
            arrays[key + "/shape"] = np.array(case["shape"], dtype=np.int64)
            arrays[key + "/kind"] = np.array({"c2c": 0, "r2c": 1, "dct2": 2}[case["kind"]], dtype=np.int64)
            arrays[key + "/output"] = np.asarray(case["output"],
                                                 dtype=np.float64 if case["kind"] == "dct2" else np.complex128)
            if "input" in case:
                arrays[key + "/input"] = np.asarray(case["input"])
    out = os.path.join(HERE, "fftw_golden.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}: {sum(len(c) for c in sets.values())} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.relpath(__file__)} <vkfft-rs checkout>")
    main(sys.argv[1])
