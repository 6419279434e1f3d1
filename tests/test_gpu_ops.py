"""Op-level parity of the CUDA kernels against the CPU oracle (through the C ABI).

Bar: Q8 activations (q, d, sum) and matvec outputs are bit-identical to the
oracle's restatement of Q8Act::prepare and lanes::* (rust/pocketinfer/src/
quant_int.rs:17-56, 282-419) on the same inputs.
"""
import os

import numpy as np
import pytest

from pocketinfer import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
THREADS = max(1, min(32, os.cpu_count() or 1))
TYPES = [synth.Q4_K, synth.Q6_K, synth.Q8_0, synth.Q4_0]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gpu_q8(pk, x, k, b):
    act = pk.q8_quantize(dev(x.astype(np.float32)), k, b)
    torch.cuda.synchronize()
    return act, act.q.cpu().numpy(), act.d.cpu().numpy(), act.sum.cpu().numpy()


PATHS = ["mma.sync", "tcgen05"]


@pytest.fixture
def matmul_path(pk, request):
    """Runs the test with the b > 8 matvec kernel the parameter names, then
    puts the default (mma.sync) back."""
    pk.set_matmul_path(request.param)
    yield request.param
    pk.set_matmul_path("mma.sync")


def check_q8(pk, oracle, x, k, b):
    _, q, d, s = gpu_q8(pk, x, k, b)
    ref = oracle.Q8Act(x, k, b)
    assert np.array_equal(q, ref.q)
    assert np.array_equal(bits(d), bits(ref.d))
    assert np.array_equal(s, ref.sum)


@pytest.mark.parametrize("b", [1, 5, 32])
def test_q8_quantize_bitexact_random(pk, oracle, b):
    k = 2304
    x = synth.normal_f32(100 + b, k * b) * np.float32(3.0)
    check_q8(pk, oracle, x, k, b)


def test_q8_quantize_edge_values(pk, oracle):
    k = 512
    x = np.array([((i % 73) - 36.0) * 0.0625 for i in range(k)], np.float32)  # simd_q8.rs:60
    x[0], x[1], x[2] = 127.0, 0.5, -0.5
    x[32:64] = 0.0                                   # all-zero block: d = 0, inv = 0
    x[64:96] = np.float32(1e-40)                     # subnormal amax
    x[96:128] = np.linspace(-1e30, 1e30, 32, dtype=np.float32)
    x[128:160] = np.float32(-0.0)
    x[160] = np.float32(127.0 / 254.0)
    check_q8(pk, oracle, x, k, 1)


def test_q8_quantize_nonfinite(pk, oracle):
    k = 96
    x = synth.normal_f32(7, k)
    x[3] = np.nan                  # NaN is skipped by amax and quantises to 0
    x[40] = np.inf                 # inf amax -> inv 0 -> NaN products -> 0
    x[70] = -np.inf
    check_q8(pk, oracle, x, k, 1)


def oracle_matmul(oracle, t, w, k, rows, act):
    rb = oracle.row_bytes(t, k)
    return oracle.matmul(t, w, rb, k, np.zeros(1, np.float32), act.b, rows, act, threads=THREADS)


def random_rows(t, k, rows, seed):
    spec = {synth.Q4_K: synth.SPEC_Q4K, synth.Q6_K: synth.SPEC_Q6K, synth.Q8_0: synth.SPEC_Q8_0,
            synth.Q4_0: synth.SPEC_Q4_0}[t]
    return synth.quant_blocks(spec, seed, rows, k)


@pytest.mark.parametrize("matmul_path", PATHS, indirect=True)
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("b", [1, 3, 32, 40])
def test_matvec_bitexact(pk, oracle, t, b, matmul_path):
    k, rows = 1024, 96
    w = random_rows(t, k, rows, 1000 + t + b)
    x = synth.normal_f32(2000 + b, k * b)
    act_gpu, *_ = gpu_q8(pk, x, k, b)
    want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, b))
    got_raw = pk.matmul(t, dev(w), k, rows, act_gpu).cpu().numpy()
    packed = pk.pack_weights(t, dev(w), k, rows)
    got_packed = pk.matmul_packed(t, packed, k, rows, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got_raw), bits(want))
    assert np.array_equal(bits(got_packed), bits(want))


@pytest.mark.parametrize("matmul_path", PATHS, indirect=True)
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("k,rows,b", [(16384, 96, 32), (4096, 3072, 32), (4096, 8192, 20)])
def test_matvec_lanes_slices_and_chunks(pk, oracle, t, k, rows, b, matmul_path):
    """Multi-lane matvec with each tile's k range split over four warps
    (few tiles) or kept in one (many tiles), rows staged in one or several
    chunks: bit-identical to the reference order in every case."""
    w = random_rows(t, k, rows, 3000 + t + rows)
    x = synth.normal_f32(4000 + k, k * b)
    act_gpu, *_ = gpu_q8(pk, x, k, b)
    want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, b))
    got = pk.matmul(t, dev(w), k, rows, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("matmul_path", PATHS, indirect=True)
@pytest.mark.parametrize("t", [synth.Q8_0, synth.Q4_0])
@pytest.mark.parametrize("k", [160, 5760])
def test_matvec_partial_stage(pk, oracle, t, k, matmul_path):
    """32-element block types whose k is not a multiple of 256: the tcgen05
    path's last stage holds fewer than eight blocks (the M26 ffn_down has 180)."""
    rows, b = 200, 32
    w = random_rows(t, k, rows, 5000 + t + k)
    x = synth.normal_f32(6000 + k, k * b)
    act_gpu, *_ = gpu_q8(pk, x, k, b)
    want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, b))
    got = pk.matmul(t, dev(w), k, rows, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("matmul_path", PATHS, indirect=True)
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("b", [4, 24])
def test_matvec_fully_random_bytes(pk, oracle, t, b, matmul_path):
    """Every byte random (scales included), as in tests/quant_layout.rs:242-286;
    b = 4 always runs the mma.sync tiles, b = 24 the selected path."""
    k, rows = 512, 64
    be, bb = oracle.type_block(t)
    w2 = synth.random_bytes(31 + t, rows * oracle.row_bytes(t, k)).reshape(-1, bb)
    w2[:, 0:2] = np.frombuffer(np.uint16(0x3200).tobytes(), np.uint8)  # finite f16 scales
    if t == synth.Q4_K:
        w2[:, 2:4] = np.frombuffer(np.uint16(0x2C00).tobytes(), np.uint8)
    if t == synth.Q6_K:
        w2[:, 208:210] = np.frombuffer(np.uint16(0x3200).tobytes(), np.uint8)
    w = w2.reshape(-1)
    x = synth.uniform_f32(99, k * b, -1.0, 1.0)
    act_gpu, *_ = gpu_q8(pk, x, k, b)
    want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, b))
    got = pk.matmul(t, dev(w), k, rows, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


def test_config1_q4k_6144x2048(pk, oracle):
    """Q4_K 6144 x 2048, seed 0, x ~ N(0,1)."""
    w, x = synth.config1_inputs(0)
    act_gpu, *_ = gpu_q8(pk, x, 2048, 1)
    want = oracle_matmul(oracle, synth.Q4_K, w, 2048, 6144, oracle.Q8Act(x, 2048, 1))
    got = pk.matmul(synth.Q4_K, dev(w), 2048, 6144, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))
    # and close to the x86 f32 path (int8 activation rounding is the only difference)
    rb = oracle.row_bytes(synth.Q4_K, 2048)
    f = np.array([oracle.dot_row(synth.Q4_K, w[r * rb:(r + 1) * rb], 2048, x) for r in range(0, 6144, 64)])
    assert np.max(np.abs(got[::64] - f)) <= 0.02 * np.std(f)


@pytest.mark.parametrize("t", [synth.Q6_K, synth.Q4_0, synth.Q8_0])
@pytest.mark.parametrize("k,rows", synth.CONFIG2_SHAPES)
def test_config2_sweep(pk, oracle, t, k, rows):
    """Q6_K / Q4_0 / Q8_0 at the four sweep shapes, b = 1."""
    w, x = synth.config2_inputs(t, k, rows, 0)
    act_gpu, *_ = gpu_q8(pk, x, k, 1)
    want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, 1))
    packed = pk.pack_weights(t, dev(w), k, rows)
    got = pk.matmul_packed(t, packed, k, rows, act_gpu).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


def test_reference_kats_on_gpu(pk, oracle):
    """tests/quant_layout.rs:50-135 known answers, through the device path."""
    def run(t, w, x):
        k = x.size
        act, *_ = gpu_q8(pk, x, k, 1)
        return float(pk.matmul(t, dev(w), k, 1, act).cpu().numpy()[0])

    w = np.zeros(34, np.uint8)
    w[0:2] = [0x00, 0x3C]
    w[2:34] = np.arange(32)
    assert abs(run(synth.Q8_0, w, np.ones(32, np.float32)) - sum(range(32))) < 0.5
    w = np.zeros(18, np.uint8)
    w[0:2] = [0x00, 0x3C]
    w[2:18] = 0x99
    assert abs(run(synth.Q4_0, w, np.ones(32, np.float32)) - 32.0) < 0.5
    w = np.zeros(144, np.uint8)
    w[0:2] = [0x00, 0x3C]
    w[2:4] = [0x00, 0x3C]
    w[4], w[8] = 1, 2
    w[16:144] = 0x21
    x = np.array([0.25 + (j % 7) * 0.01 for j in range(256)], np.float32)
    want = oracle.dot_row(synth.Q4_K, w, 256, x)
    assert abs(run(synth.Q4_K, w, x) - want) <= abs(want) * 0.02 + 1.0
    w = np.zeros(210, np.uint8)
    w[0:128], w[128:192], w[192:208] = 0x95, 0x1B, 2
    w[208:210] = [0x00, 0x3C]
    x = np.array([0.5 + (j % 5) * 0.02 for j in range(256)], np.float32)
    want = oracle.dot_row(synth.Q6_K, w, 256, x)
    assert abs(run(synth.Q6_K, w, x) - want) <= abs(want) * 0.02 + 1.0


def test_backend_selftest_and_matvec(pk, oracle):
    """backend/opencl.rs:391-500 surface: host weights, host x/out, cached uploads."""
    be = pk.Backend(0)
    be.selftest()
    assert be.supports(synth.Q4_K) and not be.supports(synth.F32)
    k, rows = 2304, 300
    keep = []  # the weight cache is keyed by (host pointer, length), as in opencl.rs:439-460,
    for t in TYPES:  # so every host slice must stay alive while the backend can see it
        w = random_rows(t, k, rows, 555 + t)
        keep.append(w)
        x = synth.normal_f32(556, k)
        got = be.matvec(t, w, k, x, rows)
        again = be.matvec(t, w, k, x, rows)  # served from the weight cache
        want = oracle_matmul(oracle, t, w, k, rows, oracle.Q8Act(x, k, 1))
        assert np.array_equal(bits(got), bits(want))
        assert np.array_equal(bits(again), bits(want))
    be.close()


def test_op_errors(pk):
    x = dev(np.zeros(64, np.float32))
    with pytest.raises(pk.PkError) as e:
        pk.q8_quantize(dev(np.zeros(40, np.float32)), 40, 1)
    assert e.value.code == 1
    act = pk.q8_quantize(x, 64, 1)
    with pytest.raises(pk.PkError) as e:
        pk.matmul(synth.F32, dev(np.zeros(256, np.uint8)), 64, 1, act)
    assert e.value.code == 2
    with pytest.raises(pk.PkError) as e:
        pk.matmul(synth.Q4_K, dev(np.zeros(144, np.uint8)), 64, 1, act)  # k not a multiple of 256
    assert e.value.code == 1


def test_device_expf_matches_c_library(pk, oracle):
    """The softmax/SwiGLU exp returns the C library's expf bits (f32::exp in the reference)."""
    bits_all = np.arange(0, 1 << 32, 61, dtype=np.uint64).astype(np.uint32)  # ~70M patterns
    x = bits_all.view(np.float32)
    x = x[~np.isnan(x)]
    hard = np.array([float.fromhex("0x1.04845ep+5"), float.fromhex("-0x1.f8cbb2p+5"), 88.72283,
                     -103.97208, -87.33655, 0.0, -0.0, np.inf, -np.inf], np.float32)
    x = np.concatenate([hard, x])
    got = pk.expf(dev(x)).cpu().numpy()
    want = oracle.expf_batch(x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n,temp,top_p", [(1000, 0.7, 0.9), (73448, 1.0, 0.9), (73448, 0.8, 1.0), (5000, 1.3, 0.5),
                                          (5000, 1.0, 0.0), (3000, 0.5, 0.999), (1, 1.0, 0.9)])
def test_sample_matches_reference(pk, oracle, n, temp, top_p):
    """sampler.rs:21-92 with temp > 0 on the device: the same token and the same
    Rng state as the reference's sampler on the same logits (ties in the top-p
    sort included)."""
    r = oracle.Rng(7 + n)
    for trial in range(4):
        x = synth.normal_f32(100 + trial + n, n) * np.float32(3.0)
        if trial == 1 and n > 8:
            x[::7] = x[3]  # many equal probabilities
        before = r.s.value
        want = oracle.sample(x.copy(), temp, top_p, r)
        got, after = pk.sample(dev(x), temp, top_p, before)
        assert got == want and after == r.s.value


def test_sample_nonfinite_logits(pk, oracle):
    """A NaN or +inf logit makes the sum NaN: token 0 and no draw (sampler.rs:45-47)."""
    for bad in (np.nan, np.inf):
        x = synth.normal_f32(5, 500)
        x[17] = bad
        r = oracle.Rng(3)
        before = r.s.value
        want = oracle.sample(x.copy(), 1.0, 0.9, r)
        got, after = pk.sample(dev(x), 1.0, 0.9, before)
        assert got == want == 0 and after == before == r.s.value
