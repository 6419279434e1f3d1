"""pk_matmul_noalloc, the matvec for hosts that cannot allocate device memory
mid-request, through the C ABI.

Some callers hand a GPU's free memory to their own arena when they start (a
serving process that fills HBM with KV pages, for example) or run where a
stream-ordered allocation may fail; pk_matmul_noalloc packs into a fixed
scratch array inside the library instead of a temporary.  These tests check
that its results are the reference's bits (the CPU oracle) and pk_matmul's on
two calls in a row, that those calls allocate nothing, that the scratch is
already reserved once an engine exists on the device (a fresh process,
lazy module loading), and that sizes beyond the scratch are refused.

Collected last (file name) so it also runs after every other GPU test has
used the library on this device; it passes alone as well.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from pocketinfer import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SPECS = {synth.Q4_K: synth.SPEC_Q4K, synth.Q6_K: synth.SPEC_Q6K, synth.Q8_0: synth.SPEC_Q8_0,
         synth.Q4_0: synth.SPEC_Q4_0}
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pool_used():
    """(UsedMemCurrent, UsedMemHigh) of the device's default stream-ordered pool."""
    from cuda.bindings import runtime as rt

    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    vals = []
    for attr in (rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh):
        err, v = rt.cudaMemPoolGetAttribute(pool, attr)
        assert err == rt.cudaError_t.cudaSuccess
        vals.append(int(v))
    return pool, vals[0], vals[1]


def reset_pool_high(pool):
    from cuda.bindings import driver as drv
    from cuda.bindings import runtime as rt

    (err,) = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh, drv.cuuint64_t(0))
    assert err == rt.cudaError_t.cudaSuccess


@pytest.mark.parametrize("t,k,rows,b", [(synth.Q6_K, 2304, 2304, 1), (synth.Q8_0, 5760, 2304, 1),
                                        (synth.Q4_0, 2048, 6144, 3), (synth.Q4_K, 2304, 512, 1)])
def test_noalloc_bits_equal_oracle_and_matmul_twice(pk, oracle, t, k, rows, b):
    w_np = synth.quant_blocks(SPECS[t], 70 + t, rows, k)
    x = synth.normal_f32(80 + t, k * b)
    want = oracle.matmul(t, w_np, oracle.row_bytes(t, k), k, x, b, rows, oracle.Q8Act(x, k, b))
    w = dev(w_np)
    if t == synth.Q4_K:  # misaligned start: the Q4_K rows must go through the scratch too
        buf = torch.zeros(w.numel() + 16, dtype=torch.uint8, device="cuda")
        buf[1:1 + w.numel()] = w
        w = buf[1:1 + w.numel()]
    act = pk.q8_quantize(dev(x), k, b)
    ref = pk.matmul(t, w, k, rows, act).cpu().numpy()  # the existing entry point
    assert np.array_equal(ref.view(np.uint32), want.view(np.uint32))
    out = torch.empty(rows * b, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    pool, used0, _ = pool_used()
    reset_pool_high(pool)
    free0 = None
    for i in range(2):  # two calls in a row share the scratch
        pk.matmul_noalloc(t, w, k, rows, act, out=out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {i}"
        if i == 0:
            free0 = torch.cuda.mem_get_info()[0]
    assert torch.cuda.mem_get_info()[0] == free0  # the second call took no device memory
    _, used1, high1 = pool_used()
    assert used1 == used0 and high1 <= used0  # no stream-ordered allocation during either call


def test_noalloc_scratch_reserved_before_first_call_in_fresh_process():
    """CUDA loads modules lazily.  In a fresh process (CUDA_MODULE_LOADING
    unset) an engine reserves the scratch when it is created, so the first
    pk_matmul_noalloc takes less device memory than the scratch's size and
    the second takes none."""
    script = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{os.path.join(ROOT, 'pocket-workbench-android_b200')!r}]
        import numpy as np, torch
        import pocketinfer as pk
        from pocketinfer import synth
        eng = pk.Engine(None, n_ctx=16)
        k, rows = 2304, 2304
        w = torch.from_numpy(synth.quant_blocks(synth.SPEC_Q6K, 5, rows, k)).cuda()
        act = pk.q8_quantize(torch.from_numpy(synth.normal_f32(6, k)).cuda(), k, 1)
        out = torch.empty(rows, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        f0 = torch.cuda.mem_get_info()[0]
        pk.matmul_noalloc(synth.Q6_K, w, k, rows, act, out=out)
        torch.cuda.synchronize()
        f1 = torch.cuda.mem_get_info()[0]
        pk.matmul_noalloc(synth.Q6_K, w, k, rows, act, out=out)
        torch.cuda.synchronize()
        f2 = torch.cuda.mem_get_info()[0]
        print(f0 - f1, f1 - f2, pk.NOALLOC_SCRATCH_BYTES)
    """)
    env = {k: v for k, v in os.environ.items() if k != "CUDA_MODULE_LOADING"}
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    first, second, scratch = (int(v) for v in r.stdout.split()[-3:])
    assert first < scratch, (first, scratch)
    assert second == 0


def test_noalloc_rejects_rows_beyond_scratch(pk):
    k, rows = 2048, 65536  # Q6_K head shape: ~110 MB packed, above the 16 MiB scratch
    assert pk.lib().pk_packed_bytes(synth.Q6_K, k, rows) > pk.NOALLOC_SCRATCH_BYTES
    w = torch.zeros(rows * pk.row_bytes(synth.Q6_K, k), dtype=torch.uint8, device="cuda")
    act = pk.q8_quantize(dev(np.zeros(k, np.float32)), k, 1)
    with pytest.raises(pk.PkError) as e:
        pk.matmul_noalloc(synth.Q6_K, w, k, rows, act)
    assert e.value.code == 1 and "scratch" in str(e.value)
