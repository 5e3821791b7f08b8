"""The committed CFFI shim (clq.lisp) and the listing in INTEGRATION.md are
the same text, and the shim binds exactly the four drop-in kernels and the
release hook that include/clq.h declares (no Lisp runs here: the check is
textual)."""
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_listing_matches_the_file():
    doc = (ROOT / "INTEGRATION.md").read_text()
    m = re.search(r"## 2\. The CFFI shim[^\n]*\n\n```lisp\n(.*?)```", doc, re.S)
    assert m, "INTEGRATION.md has no shim listing"
    assert m.group(1) == (ROOT / "clq.lisp").read_text()


def test_shim_names_declared_entry_points():
    shim = (ROOT / "clq.lisp").read_text()
    header = (ROOT / "include" / "clq.h").read_text()
    names = set(re.findall(r'"(clq_[a-z0-9_]+)"', shim))
    assert names == {"clq_last_error", "clq_forget", "clq_q8_0_matmul", "clq_q4_0_matmul", "clq_q4_k_matmul",
                     "clq_q6_k_matmul"}
    for name in names:
        assert re.search(r"\bint " + name + r"\(", header), name
    # the kernel signature of the trivial-simd slot: (out x bytes M N K)
    assert "(out :pointer) (x :pointer) (bytes :pointer) (m :int64) (n :int64) (k :int64)" in shim
