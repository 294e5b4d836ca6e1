"""GPU parity of the weight-streaming GEMV programs (one persistent launch
running a dependency chain of mat-muls) against the oracle.

Every op is checked teacher-forced: the oracle mat-mul of the op's weight
applied to the op's actual device input (which, for a dependent op, was
written by an earlier op of the same launch).  Gate: pre-rounding fp32
outputs within 1e-3 relative (accumulation order), bf16 epilogues within
one bf16 ulp."""
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


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_decode_layer_chain(ctx, wtype, M):
    """q,k,v | o | gate,up | down -- the dependency groups of a decode layer,
    each reading the previous group's output."""
    H, QD, KD, F = 512, 512, 256, 1024
    if wtype == O.TYPE_F16 and M == 8:
        F = 1024      # 8 * 1024 * 2 bytes = 16 KiB operand limit
    shapes = {"q": (H, QD), "k": (H, KD), "v": (H, KD), "o": (QD, H), "gate": (H, F), "up": (H, F), "down": (F, H)}
    host_w = {n: S.weight(wtype, N, K) for n, (K, N) in shapes.items()}
    W = {n: ctx.weight(wtype, K, N, host_w[n]) for n, (K, N) in shapes.items()}
    x = torch.from_numpy(S.normal((M, H))).cuda()
    y = {n: torch.zeros((M, N), dtype=torch.float32, device="cuda") for n, (K, N) in shapes.items()}
    ops = [dict(w=W["q"], x=x, y=y["q"], M=M, group=0),
           dict(w=W["k"], x=x, y=y["k"], M=M, group=0, flags=vb.OUT_BF16),
           dict(w=W["v"], x=x, y=y["v"], M=M, group=0),
           dict(w=W["o"], x=y["q"], y=y["o"], M=M, group=1, wait_group=0),
           dict(w=W["gate"], x=y["o"], y=y["gate"], M=M, group=2, wait_group=1),
           dict(w=W["up"], x=y["o"], y=y["up"], M=M, group=2, wait_group=1, flags=vb.OUT_BF16),
           dict(w=W["down"], x=y["gate"], y=y["down"], M=M, group=3, wait_group=2)]
    prog = vb.Program(ctx, ops)
    torch.cuda.synchronize()
    for _ in range(2):   # a second run reuses the barriers (reset per run)
        prog.run()
    rc, err = prog.status()
    assert rc == 0 and err == 0, ctx.last_error()
    inputs = {"q": x, "k": x, "v": x, "o": y["q"], "gate": y["o"], "up": y["o"], "down": y["gate"]}
    for o in ops:
        name = [n for n in W if W[n] is o["w"]][0]
        K, N = shapes[name]
        ref = O.matmul(wtype, host_w[name], K, N, host(inputs[name]))
        got = host(y[name])
        if o.get("flags"):
            S.assert_layer_close(got, O.bf16_round(ref), 1e-3)
        else:
            S.assert_matmul_close(got, ref, 1e-3)
    prog.close()
    for w in W.values():
        w.release()


def test_program_matches_per_op_launch(ctx):
    """The same op through vb_matmul and through a program gives the same
    values within accumulation order (bias + bf16 epilogue included)."""
    K, N, M = 2048, 6144, 2
    hw = S.weight(O.TYPE_Q8_0, N, K)
    w = ctx.weight(O.TYPE_Q8_0, K, N, hw)
    x = torch.from_numpy(S.normal((M, K))).cuda()
    b = torch.from_numpy(S.normal(N, 0.1)).cuda()
    y1 = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    y2 = torch.zeros_like(y1)
    torch.cuda.synchronize()
    ctx.matmul(w, x, M, y1, vb.OUT_BF16, bias=b)
    prog = vb.Program(ctx, [dict(w=w, x=x, y=y2, M=M, group=0, bias=b, flags=vb.OUT_BF16)])
    prog.run()
    rc, err = prog.status()
    assert rc == 0 and err == 0
    ref = O.bf16_round(O.matmul(O.TYPE_Q8_0, hw, K, N, host(x)) + host(b))
    S.assert_layer_close(host(y2), ref, 1e-3)
    S.assert_layer_close(host(y2), host(y1), 1e-3)
    prog.close()
    w.release()


def test_f16_long_rows_split_over_warps(ctx):
    """F16 M = 1 ops whose ring chunk holds 2 or 4 rows (K 4096 / 6144 / 8192),
    so several warps share a row: ragged N (last chunks of one row, CTAs with
    no rows), bias + bf16 epilogues, and dependent ops after them on the same
    CTAs (the ring position must continue exactly where the split ops left
    it)."""
    cases = [  # K, N, bias, flags, group, wait_group, input (index of an earlier op or None)
        (6144, 2048, True, vb.OUT_BF16, 0, -1, None),
        (4096, 301, False, 0, 0, -1, None),
        (8192, 150, True, 0, 0, -1, None),
        (6144, 37, False, vb.OUT_BF16, 0, -1, None),
        (2048, 8192, False, 0, 1, 0, 0),          # F16 K = 2048 reading op 0's output
        (6144, 4096, False, 0, 2, 1, 4),          # then a long-row op reading op 4's output
    ]
    ops, keep = [], []
    for i, (K, N, has_b, flags, g, wg, src) in enumerate(cases):
        hw = S.weight(O.TYPE_F16, N, K)
        w = ctx.weight(O.TYPE_F16, K, N, hw)
        x = torch.from_numpy(S.normal((1, K))).cuda() if src is None else None
        y = torch.zeros((1, N), dtype=torch.float32, device="cuda")
        b = torch.from_numpy(S.normal(N, 0.3)).cuda() if has_b else None
        keep.append(dict(hw=hw, w=w, x=x, y=y, b=b, K=K, N=N, flags=flags, src=src))
    for i, c in enumerate(keep):
        if c["src"] is not None:
            c["x"] = keep[c["src"]]["y"][:, :c["K"]]
        K, N, has_b, flags, g, wg, _ = cases[i]
        ops.append(dict(w=c["w"], x=c["x"], y=c["y"], M=1, group=g, wait_group=wg, bias=c["b"], flags=flags))
    prog = vb.Program(ctx, ops)
    torch.cuda.synchronize()
    for _ in range(2):
        prog.run()
    rc, err = prog.status()
    assert rc == 0 and err == 0, ctx.last_error()
    for c in keep:
        ref = O.matmul(O.TYPE_F16, c["hw"], c["K"], c["N"], host(c["x"]))
        if c["b"] is not None:
            ref = ref + host(c["b"])
        if c["flags"]:
            S.assert_layer_close(host(c["y"]), O.bf16_round(ref), 1e-3)
        else:
            S.assert_matmul_close(host(c["y"]), ref, 1e-3)
    prog.close()
    for c in keep:
        c["w"].release()


def test_odd_shapes_and_scale_fallback(ctx):
    """K = 64 and 1024 (scales not bulk-copyable, read from global), N < #SMs
    (most CTAs own no rows), N not a multiple of the chunk."""
    cases = [(64, 1024), (1024, 64), (1024, 100), (96, 7)]
    ops, keep = [], []
    for i, (K, N) in enumerate(cases):
        hw = S.weight(O.TYPE_Q8_0, N, K)
        w = ctx.weight(O.TYPE_Q8_0, K, N, hw)
        x = torch.from_numpy(S.normal((1, K))).cuda()
        y = torch.zeros((1, N), dtype=torch.float32, device="cuda")
        ops.append(dict(w=w, x=x, y=y, M=1, group=i, wait_group=i - 1))
        keep.append((hw, x, y, K, N))
    prog = vb.Program(ctx, ops)
    torch.cuda.synchronize()
    prog.run()
    rc, err = prog.status()
    assert rc == 0 and err == 0
    for hw, x, y, K, N in keep:
        S.assert_matmul_close(host(y), O.matmul(O.TYPE_Q8_0, hw, K, N, host(x)), 1e-3)
    prog.close()


def test_program_rejects_bad_ops(ctx):
    hw = S.weight(O.TYPE_Q8_0, 64, 2048)
    w = ctx.weight(O.TYPE_Q8_0, 2048, 64, hw)
    x = torch.zeros((16, 2048), dtype=torch.float32, device="cuda")
    y = torch.zeros((16, 64), dtype=torch.float32, device="cuda")
    bad = [
        [dict(w=w, x=x, y=y, M=9, group=0)],                                   # M > 8
        [dict(w=w, x=x.data_ptr() + 4, y=y, M=1, group=0)],                    # misaligned x
        [dict(w=w, x=x, y=y, M=1, group=1), dict(w=w, x=x, y=y, M=1, group=0)],  # decreasing groups
        [dict(w=w, x=x, y=y, M=1, group=0, wait_group=0)],                     # waits on itself
    ]
    for ops in bad:
        with pytest.raises(vb.VBError) as e:
            vb.Program(ctx, ops)
        assert e.value.code == vb.VB_ERR_INVALID_ARG
