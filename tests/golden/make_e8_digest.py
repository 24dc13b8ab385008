"""Record the digest that identifies the reference's E8 codebook.

The reference ships the E8 codebook as a literal table (E8_I8 in
crates/uor-matmul-codec/src/e8.rs, 256 rows of 8 i8). This script reads that
table as text, packs it row-major into 2048 bytes and writes their SHA-256 to
``e8_digest.json``; the library derives the table itself and the CPU tests
compare its bytes with the digest, so no reference file is needed at test time.

Run in a container where the reference is mounted:
    python tests/golden/make_e8_digest.py <path to the uor-matmul checkout>
"""
import hashlib
import json
import pathlib
import re
import sys

HERE = pathlib.Path(__file__).parent
SOURCE = "crates/uor-matmul-codec/src/e8.rs"


def main(root):
    src = (pathlib.Path(root) / SOURCE).read_text()
    start = src.index("= [", src.index("pub static E8_I8"))
    body = src[start:src.index("\n];", start)]
    rows = [[int(x) for x in r.split(",")] for r in re.findall(r"\[([-0-9, ]+)\]", body)]
    assert len(rows) == 256 and all(len(r) == 8 for r in rows)
    data = bytes((v & 0xFF) for r in rows for v in r)
    rec = {"source": SOURCE + " (E8_I8)", "rows": 256, "block": 8,
           "sha256": hashlib.sha256(data).hexdigest()}
    (HERE / "e8_digest.json").write_text(json.dumps(rec, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "e8_digest.json")


if __name__ == "__main__":
    main(sys.argv[1])
