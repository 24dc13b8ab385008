"""Record the digests that identify the reference's committed golden vectors.

The reference commits two out-of-ecosystem NumPy oracles for this path:
CX-10 (``oracles/numpy``: int64 wrapping matmul, 8 shapes) and CX-11
(``oracles/tropical``: (max, +) over masked values, 16 shapes). Their inputs are
drawn from a recorded xorshift generator, so the parity tests regenerate them
and compare SHA-256 digests of the regenerated inputs and of the oracle's
outputs with the digests below -- no reference file is needed at test time.

Run in a container where the reference is mounted:
    python tests/golden/make_cx_manifest.py /path/to/uor-matmul
"""
import json
import pathlib
import sys

HERE = pathlib.Path(__file__).parent


def main(root):
    root = pathlib.Path(root)
    out = {}
    for key, sub in (("cx10", "numpy"), ("cx11", "tropical")):
        man = json.loads((root / "oracles" / sub / "manifest.json").read_text())
        rec = {k: man[k] for k in ("id", "seed", "dtype", "byte_order") if k in man}
        for k in ("neg_inf", "span", "mask_a", "mask_b", "semiring"):
            if k in man:
                rec[k] = man[k]
        rec["source"] = f"oracles/{sub}/manifest.json"
        rec["cases"] = [
            {"stem": c["stem"], "shape": c["shape"], "a_sha256": c["a_sha256"],
             "b_sha256": c["b_sha256"], "expected_sha256": c["expected_sha256"]}
            for c in man["cases"]
        ]
        out[key] = rec
    (HERE / "cx_manifest.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "cx_manifest.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_cx_manifest.py <path to the uor-matmul checkout>")
    main(sys.argv[1])
