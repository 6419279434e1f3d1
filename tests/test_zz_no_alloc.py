"""pk_matmul_noalloc against pk_matmul, through the C ABI.

Collected last (file name) so it also runs after every other GPU test has
used the library on this device; it passes alone as well, and then makes
the first call itself, which looks up the scratch.
"""
import numpy as np
import pytest

from pocketinfer import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SPECS = {synth.Q4_K: synth.SPEC_Q4K, synth.Q6_K: synth.SPEC_Q6K, synth.Q8_0: synth.SPEC_Q8_0,
         synth.Q4_0: synth.SPEC_Q4_0}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("t,k,rows,b", [(synth.Q6_K, 2304, 2304, 1), (synth.Q8_0, 5760, 2304, 1),
                                        (synth.Q4_0, 2048, 6144, 3), (synth.Q4_K, 2304, 512, 1)])
def test_noalloc_matches_matmul_twice(pk, t, k, rows, b):
    w = dev(synth.quant_blocks(SPECS[t], 70 + t, rows, k))
    if t == synth.Q4_K:  # misaligned start: the Q4_K rows must go through the scratch too
        buf = torch.zeros(w.numel() + 16, dtype=torch.uint8, device="cuda")
        buf[1:1 + w.numel()] = w
        w = buf[1:1 + w.numel()]
    act = pk.q8_quantize(dev(synth.normal_f32(80 + t, k * b)), k, b)
    want = pk.matmul(t, w, k, rows, act).cpu().numpy()
    for _ in range(2):  # two calls in a row reuse the same scratch
        got = pk.matmul_noalloc(t, w, k, rows, act).cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=0.0)


def test_noalloc_rejects_rows_beyond_scratch(pk):
    k, rows = 2048, 65536  # Q6_K head shape: ~110 MB packed, above the 16 MiB scratch
    assert pk.lib().pk_packed_bytes(synth.Q6_K, k, rows) > pk.NOALLOC_SCRATCH_BYTES
    w = torch.zeros(rows * pk.row_bytes(synth.Q6_K, k), dtype=torch.uint8, device="cuda")
    act = pk.q8_quantize(dev(np.zeros(k, np.float32)), k, 1)
    with pytest.raises(pk.PkError) as e:
        pk.matmul_noalloc(synth.Q6_K, w, k, rows, act)
    assert e.value.code == 1 and "scratch" in str(e.value)
