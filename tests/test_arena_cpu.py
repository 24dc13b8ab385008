"""The Arena tier's host side and its decode restatement, pinned to the reference's
CK-14 symbol corpus (oracles/symbols) by digest: canonicalize builds the codebook,
the xorshift stream gives the codes, and the oracle's decode gives the weights."""
import hashlib
import json
import os

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc

MANIFEST = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                       "ck14_manifest.json")))


def sha(x):
    return "sha256:" + hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def ck14_codebook():
    """The corpus's symbols, (q - 127.5) 2^-6 for q < 256, in the library's canonical
    order (the stream is shuffled first: the order must come from canonicalize)."""
    values = (np.arange(256, dtype=np.float32) - np.float32(127.5)) * np.float32(2.0 ** -6)
    stream = np.concatenate([values, values[::3]])  # repeats collapse
    np.random.default_rng(0).shuffle(stream)
    n = U.arena_canonicalize(stream)
    assert n == 256
    return stream[:n].copy()


def test_canonical_codebook_matches_ck14():
    assert sha(ck14_codebook().astype("<f4")) == MANIFEST["codebook_sha256"]


def ck14_codes(idx):
    s = MANIFEST["seed"]
    for case in MANIFEST["cases"][: idx + 1]:
        n, k = case["shape"]["n"], case["shape"]["k"]
        states, s = orc.xorshift_stream(s, n * k)
        codes = ((states >> np.uint64(33)) % np.uint64(256)).astype(np.uint8)
    return case, codes


@pytest.mark.parametrize("idx", range(len(MANIFEST["cases"])))
def test_codes_and_decoded_weights_match_ck14(idx):
    case, codes = ck14_codes(idx)
    n, k = case["shape"]["n"], case["shape"]["k"]
    assert sha(codes) == case["codes_sha256"]
    weights = orc.decode_arena(ck14_codebook(), codes, n, k)
    assert sha(weights.astype("<f4")) == case["weights_sha256"]


def test_canonicalize_orders_bit_patterns_without_float_comparison():
    """CK-10: unsigned order on patterns; -0.0 and +0.0 are two symbols, NaNs with
    different payloads are distinct, equal patterns collapse."""
    bits = np.array([0x80000000, 0x00000000, 0x7FC00001, 0x7FC00000, 0x3F800000, 0x80000000,
                     0xBF800000, 0x7FC00001], np.uint32)
    v = bits.view(np.float32).copy()
    n = U.arena_canonicalize(v)
    assert n == 6
    assert v.view(np.uint32)[:n].tolist() == [0x00000000, 0x3F800000, 0x7FC00000, 0x7FC00001,
                                              0x80000000, 0xBF800000]
    # the tail keeps the sorted stream's values, as the in-place compaction leaves them
    assert v.view(np.uint32)[n:].tolist() == [0x80000000, 0xBF800000]
    d = np.array([2.0, -0.0, 2.0, 0.0], np.float64)
    assert U.arena_canonicalize(d) == 3
    assert d.view(np.uint64)[:3].tolist() == [0, 0x4000000000000000, 0x8000000000000000]
    assert U.arena_canonicalize(np.zeros(0, np.float32)) == 0


def test_decode_is_modulo_n_with_u16_codes():
    table = np.array([1.5, -2.0, 3.25], np.float32)
    codes = np.array([5, 0, 1, 1, 0xFF, 0xFF], np.uint8)  # 5, 257, 65535 little-endian
    got = orc.decode_arena(table, codes, 1, 3, code_bytes=2)
    assert got.tolist() == [[table[5 % 3], table[257 % 3], table[65535 % 3]]]
