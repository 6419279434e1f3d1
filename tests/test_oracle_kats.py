"""Pins the CPU oracle against the reference's own known-answer tests.

Each test restates one test of the reference (Aleinto97/pocket-workbench-android,
rust/pocketinfer/...) with the same inputs and the same assertion, so the
oracle is checked against the reference's golden values before it is trusted
as the parity checker for the CUDA path.
"""
import struct

import numpy as np

Q4_0, Q8_0, Q4_K, Q6_K, F32 = 2, 8, 12, 14, 0


def le16(v):
    return list(struct.pack("<H", v))


class Prng:
    """tests/quant_layout.rs:137-140 (LCG)."""

    def __init__(self, s):
        self.s = s

    def __call__(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return (self.s >> 33) & 0xFFFFFFFF


def test_q6k_block_layout(oracle):  # tests/quant_layout.rs:3-24
    block = np.zeros(210, np.uint8)
    block[0] = 0x19
    block[128] = 0x55
    block[192], block[194], block[196], block[198] = 1, 2, 3, 4
    block[208:210] = le16(0x3C00)
    out = oracle.dequant_row(Q6_K, block, 256)
    q1 = ((0x19 & 0xF) | (((0x55 >> 0) & 3) << 4)) - 32
    q2 = ((0 & 0xF) | (((0x55 >> 2) & 3) << 4)) - 32
    q3 = ((0x19 >> 4) | (((0x55 >> 4) & 3) << 4)) - 32
    q4 = ((0 >> 4) | (((0x55 >> 6) & 3) << 4)) - 32
    assert out[0] == q1
    assert out[32] == 2.0 * q2
    assert out[64] == 3.0 * q3
    assert out[96] == 4.0 * q4
    assert out[1] == -32.0


def test_q4k_block_layout(oracle):  # tests/quant_layout.rs:26-39
    block = np.zeros(144, np.uint8)
    block[0:2] = le16(0x3C00)
    block[2:4] = le16(0x3C00)
    block[4] = 1
    block[8] = 0
    block[16] = 0x21
    out = oracle.dequant_row(Q4_K, block, 256)
    assert out[0] == 1.0
    assert out[1] == 0.0
    assert out[32] == 0.0


def test_f16_roundtrip(oracle):  # tests/quant_layout.rs:41-48
    for v in [0.0, 1.0, -1.0, 0.5, 0.1, 65504.0, 6.1e-5, -0.333]:
        v32 = float(np.float32(v))
        back = oracle.f16_to_f32(oracle.f32_to_f16(v32))
        assert abs(back - v32) <= abs(v32) * 1e-3 + 1e-6, (v, back)


def test_f16_decode_matches_numpy_everywhere(oracle):
    """util.rs:76-100 decodes every f16 (subnormals included) exactly."""
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(want)]))


def test_int8_q8_0_matches(oracle):  # tests/quant_layout.rs:50-66
    w = np.zeros(34, np.uint8)
    w[0:2] = le16(0x3C00)
    w[2:34] = np.arange(32)
    act = oracle.Q8Act(np.ones(32, np.float32), 32, 1)
    got = oracle.dot_row_q8(Q8_0, w, 32, act, 0)
    assert abs(got - sum(range(32))) < 0.5


def test_int8_q4_0_matches(oracle):  # tests/quant_layout.rs:68-84
    w = np.zeros(18, np.uint8)
    w[0:2] = le16(0x3C00)
    w[2:18] = 0x99
    act = oracle.Q8Act(np.ones(32, np.float32), 32, 1)
    got = oracle.dot_row_q8(Q4_0, w, 32, act, 0)
    assert abs(got - 32.0) < 0.5


def test_int8_q4k_matches_scalar(oracle):  # tests/quant_layout.rs:86-108
    w = np.zeros(144, np.uint8)
    w[0:2] = le16(0x3C00)
    w[2:4] = le16(0x3C00)
    w[4] = 1
    w[8] = 2
    w[16:144] = 0x21
    x = np.array([0.25 + (j % 7) * 0.01 for j in range(256)], np.float32)
    act = oracle.Q8Act(x, 256, 1)
    got = oracle.dot_row_q8(Q4_K, w, 256, act, 0)
    want = oracle.dot_row(Q4_K, w, 256, x)
    assert abs(got - want) <= abs(want) * 0.02 + 1.0


def test_int8_q6k_matches_scalar(oracle):  # tests/quant_layout.rs:110-135
    w = np.zeros(210, np.uint8)
    w[0:128] = 0x95
    w[128:192] = 0x1B
    w[192:208] = 2
    w[208:210] = le16(0x3C00)
    x = np.array([0.5 + (j % 5) * 0.02 for j in range(256)], np.float32)
    act = oracle.Q8Act(x, 256, 1)
    got = oracle.dot_row_q8(Q6_K, w, 256, act, 0)
    want = oracle.dot_row(Q6_K, w, 256, x)
    assert abs(got - want) <= abs(want) * 0.02 + 1.0


def test_int8_q4k_random_block(oracle):  # tests/quant_layout.rs:142-168
    r = Prng(12345)
    w = np.zeros(288 * 8, np.uint8)
    w[0:2] = le16(0x3200)
    w[2:4] = le16(0x2C00)
    for i in range(4, 288 * 8):
        w[i] = r() & 0xFF
    for blk in range(8):
        w[blk * 144:blk * 144 + 2] = le16(0x3000)
        w[blk * 144 + 2:blk * 144 + 4] = le16(0x2800)
    x = np.array([((r() % 2000) / 1000.0) - 1.0 for _ in range(2048)], np.float32)
    act = oracle.Q8Act(x, 2048, 1)
    got = oracle.dot_row_q8(Q4_K, w, 2048, act, 0)
    want = oracle.dot_row(Q4_K, w, 2048, x)
    assert abs(got - want) <= abs(want) * 0.02 + 0.01


def test_int8_q6k_random_block(oracle):  # tests/quant_layout.rs:170-192
    r = Prng(999)
    w = np.array([r() & 0xFF for _ in range(420)], np.uint8)
    w[208:210] = le16(0x3400)
    w[418:420] = le16(0x3400)
    x = np.array([((r() % 2000) / 1000.0) - 1.0 for _ in range(512)], np.float32)
    act = oracle.Q8Act(x, 512, 1)
    got = oracle.dot_row_q8(Q6_K, w, 512, act, 0)
    want = oracle.dot_row(Q6_K, w, 512, x)
    assert abs(got - want) <= abs(want) * 0.02 + 0.01


def test_row_dot_multi_matches_dot_row(oracle):  # tests/quant_layout.rs:194-224
    r = Prng(777)
    w = np.array([r() & 0xFF for _ in range(144 * 4)], np.uint8)
    for blk in range(4):
        w[blk * 144:blk * 144 + 2] = le16(0x3000)
        w[blk * 144 + 2:blk * 144 + 4] = le16(0x2800)
    k, b = 1024, 5
    xt = np.zeros(k * b, np.float32)
    for j in range(k):
        for bi in range(b):
            xt[j * b + bi] = ((r() % 2000) / 1000.0) - 1.0
    multi = oracle.row_dot_multi(Q4_K, w, k, xt, b)
    for bi in range(b):
        single = oracle.dot_row(Q4_K, w, k, xt.reshape(k, b)[:, bi].copy())
        assert abs(multi[bi] - single) <= abs(single) * 1e-4 + 1e-4


def _random_act(oracle, r, k, b):  # tests/quant_layout.rs:232-240
    x = np.array([((r() % 2000) / 1000.0) - 1.0 for _ in range(k * b)], np.float32)
    return oracle.Q8Act(x, k, b)


def _random_row(oracle, r, ttype, k):
    be, bb = oracle.type_block(ttype)
    nblk = k // be
    row = np.array([r() & 0xFF for _ in range(bb * nblk)], np.uint8)
    for blk in range(nblk):
        base = blk * bb
        row[base:base + 2] = le16(0x3200)
        if ttype == Q4_K:
            row[base + 2:base + 4] = le16(0x2C00)
        elif ttype == Q6_K:
            row[base + 208:base + 210] = le16(0x3200)
    return row


def test_int8_multi_matches_single_bitwise(oracle):  # tests/quant_layout.rs:242-286
    r = Prng(4242)
    b, k = 32, 1024
    for ttype in (Q4_0, Q8_0, Q4_K, Q6_K):
        row = _random_row(oracle, r, ttype, k)
        act = _random_act(oracle, r, k, b)
        multi = oracle.dot_row_q8_lanes(ttype, row, k, act, b)
        for lane in range(b):
            single = oracle.dot_row_q8(ttype, row, k, act, lane)
            assert abs(multi[lane] - single) <= abs(single) * 1e-5 + 1e-4


def test_int8_multi_exact_bitwise(oracle):  # tests/quant_layout.rs:327-357
    r = Prng(99)
    b, k = 32, 512
    for ttype in (Q4_K, Q6_K):
        row = _random_row(oracle, r, ttype, k)
        act = _random_act(oracle, r, k, b)
        multi = oracle.dot_row_q8_lanes(ttype, row, k, act, b)
        for lane in range(b):
            single = np.float32(oracle.dot_row_q8(ttype, row, k, act, lane))
            assert multi[lane].view(np.uint32) == single.view(np.uint32)


def test_q8_quantization_halfway_values(oracle):  # simd_q8.rs:57-80
    k = 512
    x = np.array([((i % 73) - 36.0) * 0.0625 for i in range(k)], np.float32)
    x[0], x[1], x[2] = 127.0, 0.5, -0.5
    act = oracle.Q8Act(x, k, 1)
    for blk in range(k // 32):
        s = slice(blk * 32, blk * 32 + 32)
        amax = np.float32(np.max(np.abs(x[s])))
        d = np.float32(amax / np.float32(127.0))
        inv = np.float32(np.float32(1.0) / d) if d > 0 else np.float32(0.0)
        xs = (x[s] * inv).astype(np.float32)
        q = np.clip(np.sign(xs) * np.floor(np.abs(xs) + np.float32(0.5)), -127, 127).astype(np.int32)
        assert np.array_equal(act.q[s].astype(np.int32), q)
        assert act.d[blk].view(np.uint32) == d.view(np.uint32)
        assert act.sum[blk] == q.sum()


def test_opencl_selftest_blocks(oracle):  # backend/opencl.rs:391-430 gate, int8 path vs f32 path
    k = 256
    x = np.array([(j % 7) * 0.1 - 0.3 for j in range(k)], np.float32)
    w4 = np.zeros(144, np.uint8)
    w4[0:2] = le16(0x3C00)
    w4[4] = 1
    w4[16:144] = 0x21
    act = oracle.Q8Act(x, k, 1)
    got = oracle.dot_row_q8(Q4_K, w4, k, act, 0)
    want = oracle.dot_row(Q4_K, w4, k, x)
    assert abs(got - want) <= abs(want) * 0.02 + 0.01
    w6 = np.zeros(210, np.uint8)
    w6[0:128] = 0x95
    w6[128:192] = 0x1B
    w6[192:208] = 2
    w6[208:210] = le16(0x3C00)
    got = oracle.dot_row_q8(Q6_K, w6, k, act, 0)
    want = oracle.dot_row(Q6_K, w6, k, x)
    assert abs(got - want) <= abs(want) * 0.02 + 0.01


def test_tensor_nbytes_overflow_rejected(oracle):  # quant.rs:723-731
    assert oracle.lib().pko_tensor_nbytes(F32, 2**64 - 1, 2**64 - 1) == -1
    assert oracle.lib().pko_tensor_nbytes(Q4_K, 255, 1) == -1
    assert oracle.lib().pko_tensor_nbytes(Q4_K, 2304, 2304) == 2304 * 9 * 144


def test_int_dots_reconstruct_lanes_sum(oracle):
    """The per-term integer dots, combined in the reference's order, rebuild
    lanes::* bit-for-bit (the decomposition the CUDA kernels use)."""
    r = Prng(31337)
    k = 1024

    def f16(lo, hi):
        return np.float32(np.frombuffer(bytes([lo, hi]), np.float16)[0])

    for ttype in (Q4_0, Q8_0, Q4_K, Q6_K):
        row = _random_row(oracle, r, ttype, k)
        act = _random_act(oracle, r, k, 1)
        dots = oracle.row_int_dots(ttype, row, k, act, 0)
        acc = np.float32(0.0)
        be, bb = oracle.type_block(ttype)
        if ttype in (Q4_0, Q8_0):
            for blk in range(k // 32):
                d = f16(row[blk * bb], row[blk * bb + 1])
                da = act.d[blk]
                if ttype == Q8_0:
                    t = np.float32(d * da) * np.float32(dots[blk])
                else:
                    t = np.float32(d * da) * np.float32(np.float32(dots[blk]) - np.float32(8.0) * np.float32(act.sum[blk]))
                acc = np.float32(acc + t)
        elif ttype == Q4_K:
            for blk in range(k // 256):
                b0 = blk * 144
                d, dmin = f16(row[b0], row[b0 + 1]), f16(row[b0 + 2], row[b0 + 3])
                sc = row[b0 + 4:b0 + 16]
                for sb in range(8):
                    if sb < 4:
                        s, m = sc[sb] & 63, sc[sb + 4] & 63
                    else:
                        s = (sc[sb + 4] & 0xF) | ((sc[sb - 4] >> 6) << 4)
                        m = (sc[sb + 4] >> 4) | ((sc[sb] >> 6) << 4)
                    da, sa = act.d[blk * 8 + sb], act.sum[blk * 8 + sb]
                    t1 = np.float32(np.float32(np.float32(d * da) * np.float32(s)) * np.float32(dots[blk * 8 + sb]))
                    t2 = np.float32(np.float32(np.float32(da * dmin) * np.float32(m)) * np.float32(sa))
                    acc = np.float32(acc + np.float32(t1 - t2))
        else:
            n = 0
            for blk in range(k // 256):
                b0 = blk * 210
                d = f16(row[b0 + 208], row[b0 + 209])
                for half in range(2):
                    for g in range(2):
                        for s in range(4):
                            scale = np.float32(np.int8(row[b0 + 192 + half * 8 + g + 2 * s]))
                            da = act.d[blk * 8 + 4 * half + s]
                            t = np.float32(np.float32(np.float32(d * scale) * da) * np.float32(dots[n]))
                            acc = np.float32(acc + t)
                            n += 1
        want = np.float32(oracle.dot_row_q8(ttype, row, k, act, 0))
        assert acc.view(np.uint32) == want.view(np.uint32), ttype
