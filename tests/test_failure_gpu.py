"""Failure detection on the GPU in the forms this pool allows: no fault, no
trap, no endless wait.  Every wait of the streaming kernel on other CTAs is
bounded; with the bound lowered to a few hundred cycles
(vb_set_wait_limit) a dependency cannot be met in time, so the kernel
records STREAM_TIMEOUT_GRID, stops and exits, the status call reports it as
VB_ERR_BACKEND (and clears it), and the same context, program and decoder
then run correctly again.  Host-side fault injection (VB_FAULT=launch) turns the first kernel
launch of an op into an error status without touching the device."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402

STREAM_TIMEOUT_GRID = 3
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.set_wait_limit(0)
    c.close()


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def zeros(shape):
    t = torch.zeros(shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    return t


def test_program_dependency_timeout_is_reported_and_recovers(ctx):
    """A two-group program (group 1 reads group 0's output): with a 200-cycle
    bound the CTAs that finish group 0 first cannot see every other CTA's
    arrival in time.  Afterwards, with the default bound, the same program
    gives the oracle's result."""
    K, N = 2048, 6144
    w0 = S.weight(O.TYPE_Q8_0, N, K)
    w1 = S.weight(O.TYPE_Q8_0, K, N)
    W0, W1 = ctx.weight(O.TYPE_Q8_0, K, N, w0), ctx.weight(O.TYPE_Q8_0, N, K, w1)
    x = O.bf16_round(S.normal((1, K)))
    xd, y0, y1 = dev(x), zeros((1, N)), zeros((1, K))
    prog = vb.Program(ctx, [dict(w=W0, x=xd, y=y0, M=1, group=0, flags=vb.OUT_BF16),
                            dict(w=W1, x=y0, y=y1, M=1, group=1, wait_group=0)])
    ctx.set_wait_limit(200)
    prog.run()
    rc, err = prog.status()
    assert rc == vb.VB_ERR_BACKEND and err == STREAM_TIMEOUT_GRID
    ctx.set_wait_limit(0)
    prog.run()
    rc, err = prog.status()
    assert rc == vb.VB_OK and err == 0
    r0 = O.bf16_round(O.matmul(O.TYPE_Q8_0, w0, K, N, x))
    S.assert_matmul_close(y0.cpu().numpy(), r0)
    S.assert_matmul_close(y1.cpu().numpy(), O.matmul(O.TYPE_Q8_0, w1, N, K, y0.cpu().numpy()))
    # the context still runs other work
    y2 = zeros((1, N))
    ctx.matmul(W0, xd, 1, y2, vb.OUT_BF16)
    ctx.sync()
    S.assert_layer_close(y2.cpu().numpy(), y0.cpu().numpy())
    prog.close()
    W0.release()
    W1.release()


def test_decoder_step_timeout_is_reported_and_recovers(ctx):
    """The single-launch decode step with a 100-cycle bound times out on its
    first cross-CTA wait; the status reports it, and after rewinding the KV
    slot the decoder's next step equals the per-op path's."""
    H, NH, NKV, HD, F, NL = 512, 4, 2, 128, 1024, 2
    S.reseed(9100)
    layers = [S.layer(O.TYPE_Q8_0, H, NH, NKV, HD, F) for _ in range(NL)]
    fn = S.normal(H, 0.02, 1.0)
    cfg = vb.LMConfig(H, NH, NKV, HD, F, NL, 1e-5, 10000.0, 0, 0.0, O.TYPE_Q8_0)
    lm = vb.LM(ctx, cfg, layers, fn)
    kv = vb.KV(ctx, lm, 2, 64)
    T = 5
    p1 = O.bf16_round(S.normal((T, H)))
    prompt = dev(np.stack([p1, p1]))     # both slots hold the same prompt
    x = dev(O.bf16_round(S.normal((1, H))))
    pre = zeros((2, T, H))
    lm.forward(kv, [0, 1], [0, 0], T, prompt, pre)
    dec = vb.Decoder(ctx, lm, kv, [0])
    a = zeros((1, H))
    ctx.set_wait_limit(100)
    dec.step([T], x, a)
    rc, err = dec.status()
    assert rc == vb.VB_ERR_BACKEND and err == STREAM_TIMEOUT_GRID
    ctx.set_wait_limit(0)
    # rewind slot 0 to the prompt and step again
    kv.reset(0)
    lm.forward(kv, [0], [0], T, prompt[0], pre[0])
    dec.step([T], x, a)
    rc, err = dec.status()
    assert rc == vb.VB_OK and err == 0
    b = zeros((1, H))
    lm.forward(kv, [1], [T], 1, x, b)
    ctx.sync()
    S.assert_layer_close(a.cpu().numpy(), b.cpu().numpy(), tol=1e-2)
    assert kv.used(0) == T + 1 and kv.used(1) == T + 1
    dec.close()
    kv.close()
    lm.close()


def test_injected_launch_fault_is_a_status():
    """VB_FAULT=launch: the first launch check of an op reports
    VB_ERR_BACKEND with the injected message, in a child process."""
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import numpy as np, torch, vcpm_b200 as vb, oracle as O\n"
        "c = vb.Context(0)\n"
        "w = c.weight(O.TYPE_Q8_0, 64, 32, O.make_weight(O.TYPE_Q8_0, np.ones((32, 64), np.float32), O.QRULE_REF))\n"
        "x = torch.ones(1, 64, device='cuda'); y = torch.zeros(1, 32, device='cuda'); torch.cuda.synchronize()\n"
        "rc = c.L.vb_matmul(c.h, w.h, x.data_ptr(), 1, y.data_ptr(), 0)\n"
        "print(rc, c.last_error())\n"
    ) % (os.path.join(ROOT, "voxcpm-cpp_b200"), os.path.join(ROOT, "oracle"))
    env = dict(os.environ, VB_FAULT="launch")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    rc, msg = out.stdout.strip().split(" ", 1)
    assert int(rc) == vb.VB_ERR_BACKEND and "injected launch fault" in msg
