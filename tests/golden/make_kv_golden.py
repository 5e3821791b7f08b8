"""Regenerate tests/golden/kv_golden.json from the cl-inference sources.

Reads, as text, the Q8 KV-cache cases of the reference's
tests/local/cache.lisp:
  * q8-cache-groups-rounding-and-overwrite: the 35-wide row (seven listed
    values, then zeros) and the decoded row the test expects, the cache's
    byte and scale counts for three positions, and the all-zero group's scale;
  * q8-cache-reconstructs-finite-extrema: the row (most-positive-single-float,
    -most-positive-single-float) decodes to itself;
  * q8-cache-encodes-strided-rows: (arange 210) as (2 3 35), axes (1 0 2);
  * q8-cache-rejects-nonfinite-values-and-invalid-options: +inf and NaN rows.
Values are written as decimal floats; the extrema as the names the test uses.

Usage: python tests/golden/make_kv_golden.py /path/to/cl-inference
Only this script reads the reference checkout; tests read the JSON it writes.
"""
import json
import pathlib
import re
import sys

HERE = pathlib.Path(__file__).resolve().parent


def lisp_number(token):
    return float(token.replace("f", "e").replace("d", "e"))


def lisp_list(text):
    """The values of a Lisp list literal body such as '127f0 -127f0 0.5f0'."""
    return [lisp_number(t) for t in text.split()]


def parse(text):
    test = re.search(r"\(test q8-cache-groups-rounding-and-overwrite(.*?)\n\(test ", text, re.S).group(1)
    # (append '(...) (make-list 25 :initial-element 0f0) '(0f0 0f0 0f0))
    head = re.search(r"\(append '\(([^)]*)\)\s*\(make-list (\d+) :initial-element ([^)]*)\)\s*'\(([^)]*)\)\)",
                     test, re.S)
    row = lisp_list(head.group(1)) + [lisp_number(head.group(3))] * int(head.group(2)) + lisp_list(head.group(4))
    dims = [int(v) for v in re.search(r"\(ct:reshape \(ct:from-data values\) '\(([^)]*)\)\)", test).group(1).split()]
    n_ctx = int(re.search(r"\(local:make-kv-cache (\d+) :cache-type :q8\)", test).group(1))
    want = re.search(r"\(list \(append '\(([^)]*)\)\s*\(make-list (\d+) :initial-element ([^)]*)\)\)\)", test, re.S)
    decoded = lisp_list(want.group(1)) + [lisp_number(want.group(3))] * int(want.group(2))
    n_bytes = int(re.search(r"\(= (\d+) \(length \(local::q8-buffer-bytes keys\)\)\)", test).group(1))
    n_scales = int(re.search(r"\(= (\d+) \(length \(local::q8-buffer-scales keys\)\)\)", test).group(1))
    zero_scale = re.search(r"\(= ([^ ]+) \(aref \(local::q8-buffer-scales keys\) (\d+)\)\)", test)
    strided = re.search(r"\(test q8-cache-encodes-strided-rows(.*?)\n\(test ", text, re.S).group(1)
    arange = int(re.search(r"\(ct:arange (\d+)\)", strided).group(1))
    shape = [int(v) for v in re.search(r"\(ct:arange \d+\) '\(([^)]*)\)\)", strided).group(1).split()]
    axes = [int(v) for v in re.search(r":axes '\(([^)]*)\)", strided).group(1).split()]
    extrema = re.search(r"\(test q8-cache-reconstructs-finite-extrema(.*?)\n\(defun ", text, re.S).group(1)
    assert "most-positive-single-float" in extrema
    nonfinite = re.search(r"\(dolist \(name '\(([^)]*)\)\)", text).group(1).split()
    return {
        "rounding": {"row": row, "shape": dims, "n_ctx": n_ctx, "decoded": decoded, "bytes": n_bytes,
                     "scales": n_scales, "zero_group_scale": lisp_number(zero_scale.group(1)),
                     "zero_group_index": int(zero_scale.group(2))},
        "strided": {"arange": arange, "shape": shape, "axes": axes},
        "extrema": {"row": ["most-positive-single-float", "-most-positive-single-float"]},
        "nonfinite": [n.split(":")[-1] for n in nonfinite],
        "source": "tests/local/cache.lisp",
    }


def main():
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {sys.argv[0]} /path/to/cl-inference")
    root = pathlib.Path(sys.argv[1])
    text = (root / "tests" / "local" / "cache.lisp").read_text()
    out = parse(text)
    (HERE / "kv_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {HERE / 'kv_golden.json'}")


if __name__ == "__main__":
    main()
