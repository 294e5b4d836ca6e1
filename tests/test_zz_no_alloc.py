"""GPU test of vb_attention_noalloc, the attention entry point for callers
that cannot let the library allocate device memory (a host whose own
allocator already owns the GPU's memory, or a real-time thread that cannot
risk the synchronisation of cudaMalloc).  It keeps its partial results in a
fixed array compiled into the library instead of a grown buffer.

Two calls in a row, through the C ABI, must agree with vb_attention on the
same inputs within the attention tolerance of the other tests (1e-3
relative); the second call is narrower than the first, so stale partials
left in the shared array by the first call must not leak into it.  A call
larger than the array must fail with VB_ERR_INVALID_ARG.  The file is named
to be collected last and works alone in a fresh process."""
import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def bf16_bits(a):
    return (O.bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


def make_case(L, T, nh=16, nkv=2, hd=128):
    k = O.bf16_round(S.normal((L, nkv, hd)))
    v = O.bf16_round(S.normal((L, nkv, hd)))
    q = O.bf16_round(S.normal((T, nh, hd)))
    lens = np.array([max(1, L - 3 * t) for t in range(T)], np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return dict(q=dev(q), k=dev(bf16_bits(k.transpose(1, 0, 2))), v=dev(bf16_bits(v.transpose(1, 0, 2))),
                start=dev(np.zeros(T, np.int32)), len=dev(lens), L=L, T=T, nh=nh, nkv=nkv, hd=hd)


def run_both(ctx, c):
    shape = (c["T"], c["nh"] * c["hd"])
    ref = torch.zeros(shape, dtype=torch.float32, device="cuda")
    got = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
    args = (c["L"], c["T"], c["nh"], c["nkv"], c["hd"], c["start"], c["len"])
    torch.cuda.synchronize()
    ctx.attention(c["q"], c["k"], c["v"], *args, ref)
    ctx.attention_noalloc(c["q"], c["k"], c["v"], *args, got)
    ctx.sync()
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_matches_vb_attention_twice(ctx):
    # first call: 1000 rows = 16 chunks, 3 tokens; second: 300 rows = 5 chunks
    for L, T in ((1000, 3), (300, 2)):
        got, ref = run_both(ctx, make_case(L, T))
        assert np.isfinite(got).all()
        S.assert_matmul_close(got, ref, 1e-3)


def test_noalloc_single_chunk_and_oversize(ctx):
    got, ref = run_both(ctx, make_case(40, 2))      # one chunk: no scratch used
    S.assert_matmul_close(got, ref, 1e-3)
    big = make_case(8192, 8)                         # 8 tokens x 16 heads x 128 chunks: > 4 MiB
    out = torch.zeros((8, 16 * 128), dtype=torch.float32, device="cuda")
    with pytest.raises(vb.VBError) as e:
        ctx.attention_noalloc(big["q"], big["k"], big["v"], 8192, 8, 16, 2, 128, big["start"], big["len"], out)
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    assert "scratch" in ctx.last_error()
