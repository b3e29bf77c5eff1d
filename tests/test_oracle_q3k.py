"""The Q3_K restatement in the oracle (f3), checked without a GPU.

The reference holds only Q3_K's geometry (GGML type 11, 110 bytes per 256
values: har/crates/har-model/src/lib.rs:591,
benchmarks/local-bench/crates/lb-model/src/lib.rs:84) and no arithmetic, so
there are no reference vectors: parity is unpinned.  These tests pin the
oracle's decoding to the GGUF layout it restates with hand-built blocks
(every field placed by an independent packer written here) and with a second,
pure-numpy decoder of the same layout on random blocks.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "oracle"))
import haro  # noqa: E402


def pack_scales(sc16):
    """16 six-bit scales -> 12 bytes: low nibbles of scales 0..7 / 8..15 in the
    low / high nibbles of bytes 0..7, top two bits of scale s in byte 8 + s % 4
    at bit 2 * (s // 4)."""
    b = np.zeros(12, np.uint8)
    for s, v in enumerate(sc16):
        assert 0 <= v < 64
        if s < 8:
            b[s] |= v & 15
        else:
            b[s - 8] |= (v & 15) << 4
        b[8 + s % 4] |= ((v >> 4) & 3) << (2 * (s // 4))
    return b


def make_block(d, sc16, hmask, qs):
    blk = np.zeros(110, np.uint8)
    blk[0:32] = hmask
    blk[32:96] = qs
    blk[96:108] = pack_scales(sc16)
    blk[108:110] = np.array([d], np.float16).view(np.uint8)
    return blk


def numpy_decode(blk):
    """The layout decoded a second way: the 3-bit code of value 128n + 32j + l
    is bits 2j..2j+1 of qs[32n + l] plus bit 4n + j of hmask[l] (set = no -4)."""
    d = np.frombuffer(blk[108:110].tobytes(), np.float16)[0].astype(np.float32)
    scb = blk[96:108]
    out = np.empty(256, np.float32)
    for i in range(256):
        n, j, l = i // 128, (i // 32) % 4, i % 32
        s = 8 * n + 2 * j + l // 16
        low = (scb[s] & 15) if s < 8 else (scb[s - 8] >> 4)
        high = (scb[8 + s % 4] >> (2 * (s // 4))) & 3
        scale = int(low) | (int(high) << 4)
        q2 = (int(blk[32 + 32 * n + l]) >> (2 * j)) & 3
        h = (int(blk[l]) >> (4 * n + j)) & 1
        q = q2 - (0 if h else 4)
        out[i] = np.float32(d * np.float32(scale - 32)) * np.float32(q)
    return out


def test_scale_unpacking_round_trips():
    rng = np.random.default_rng(3)
    for _ in range(20):
        sc = rng.integers(0, 64, 16)
        packed = pack_scales(sc)
        assert [haro.q3k_scale(packed, s) for s in range(16)] == list(sc)


def test_codes_follow_the_two_bit_planes_and_the_high_mask():
    sc = [33] * 16  # scale 1
    # qs bytes 0b11100100: bits 2j..2j+1 = j
    blk = make_block(1.0, sc, np.full(32, 0xFF, np.uint8), np.full(64, 0xE4, np.uint8))
    w = haro.q3k_dequant_block(blk)
    assert np.array_equal(w, np.repeat(np.tile(np.arange(4, dtype=np.float32), 2), 32))
    # no high bits: every code loses 4
    blk = make_block(1.0, sc, np.zeros(32, np.uint8), np.full(64, 0xE4, np.uint8))
    w = haro.q3k_dequant_block(blk)
    assert np.array_equal(w, np.repeat(np.tile(np.arange(4, dtype=np.float32) - 4, 2), 32))
    # the high bit of value (n, j, l) is bit 4n + j of hmask[l]
    for n in range(2):
        for j in range(4):
            blk = make_block(1.0, sc, np.full(32, 1 << (4 * n + j), np.uint8), np.zeros(64, np.uint8))
            w = haro.q3k_dequant_block(blk)
            want = np.full(256, -4.0, np.float32)
            want[128 * n + 32 * j: 128 * n + 32 * j + 32] = 0.0
            assert np.array_equal(w, want), (n, j)


def test_sub_block_scales_and_d():
    sc = list(range(20, 36))  # sub-block s has scale 20 + s, i.e. s - 12 after the -32
    blk = make_block(0.5, sc, np.full(32, 0xFF, np.uint8), np.full(64, 0x55, np.uint8))  # q = 1
    w = haro.q3k_dequant_block(blk)
    want = np.array([0.5 * (sc[8 * (i // 128) + 2 * ((i // 32) % 4) + (i % 32) // 16] - 32)
                     for i in range(256)], np.float32)
    assert np.array_equal(w, want)


def test_random_blocks_match_a_second_decoder_and_the_dot():
    w = haro.random_q3k(11, 4, 512)
    rng = np.random.default_rng(12)
    x = rng.standard_normal(512).astype(np.float32)
    got = haro.q3k_matvec(w, 4, 512, x)[0]
    for r in range(4):
        dec = np.concatenate([numpy_decode(w[r, b * 110:(b + 1) * 110]) for b in range(2)])
        assert np.array_equal(dec, np.concatenate([haro.q3k_dequant_block(w[r, b * 110:(b + 1) * 110])
                                                   for b in range(2)]))
        ref = float(np.dot(dec.astype(np.float64), x.astype(np.float64)))
        assert abs(got[r] - ref) <= 1e-5 * max(1.0, abs(ref)), (r, got[r], ref)
