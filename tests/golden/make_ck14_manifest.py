"""Record the digests that identify the reference's CK-14 symbol corpus.

The reference commits an Arena fixture (``oracles/symbols``): a 256-symbol f32
codebook in canonical arena order, u8 codes for two n x k shapes drawn from its
xorshift generator, and the dense weights those codes decode to. This script copies
the seed, shapes and SHA-256 digests from that fixture's manifest into
``ck14_manifest.json``; the tests regenerate codebook, codes and weights and compare
digests, so no reference file is needed at test time.

Run in a container where the reference is mounted:
    python tests/golden/make_ck14_manifest.py <path to the uor-matmul checkout>
"""
import json
import pathlib
import sys

HERE = pathlib.Path(__file__).parent


def main(root):
    man = json.loads((pathlib.Path(root) / "oracles" / "symbols" / "manifest.json").read_text())
    rec = {k: man[k] for k in ("id", "seed", "dtype", "byte_order", "codebook_symbols",
                               "codebook_sha256")}
    rec["source"] = "oracles/symbols/manifest.json"
    rec["cases"] = [{"stem": c["stem"], "shape": c["shape"], "codes_sha256": c["codes_sha256"],
                     "weights_sha256": c["weights_sha256"]} for c in man["cases"]]
    (HERE / "ck14_manifest.json").write_text(json.dumps(rec, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "ck14_manifest.json")


if __name__ == "__main__":
    main(sys.argv[1])
