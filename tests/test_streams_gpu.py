"""Library calls on non-default streams: repeated forward / backward / paged / decode calls
on side streams give the default-stream results, and the process exits cleanly (the
library binds the stream's context through driver entry points whose signatures must
match the requested versions; a mismatch corrupts host memory and shows at exit)."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

SCRIPT = textwrap.dedent("""
    import torch
    import tilelang_fa_v100 as fa
    from tilelang_fa_v100 import _ext
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    mk = lambda *s: torch.randn(*s, generator=g, device=dev).to(torch.bfloat16)
    q, k, v, do = mk(2, 300, 8, 128), mk(2, 300, 2, 128), mk(2, 300, 2, 128), mk(2, 300, 8, 128)
    def step():
        qq, kk, vv = (x.detach().requires_grad_(True) for x in (q, k, v))
        out = fa.tilelang_flash_attn_func(qq, kk, vv, causal=True)
        out.backward(do)
        return [out.detach(), qq.grad, kk.grad, vv.grad]
    ref = step()
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(dev) for _ in range(3)]
    for i in range(8):
        s = streams[i % 3]
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            got = step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b), "side-stream result differs"
    kc, vc = mk(40, 16, 2, 128), mk(40, 16, 2, 128)
    bt = torch.randperm(40, device=dev).to(torch.int32).view(2, 20)
    sl = torch.tensor([300, 17], dtype=torch.int32, device=dev)
    with torch.cuda.stream(streams[1]):
        for _ in range(4):
            o = fa.tilelang_decode_forward(mk(2, 8, 128), kc, vc, bt, sl)
            qp = mk(317, 8, 128)
            qsl = torch.tensor([0, 300, 317], dtype=torch.int32, device=dev)
            po, _ = fa.tilelang_paged_forward(qp, kc, vc, bt, sl, qsl, sl - torch.diff(qsl))
    torch.cuda.synchronize()
    assert _ext.read_device_error() == (0, 0, 0)
    print("side streams ok")
""")


def test_side_streams_and_clean_exit(cuda_dev):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "tilelang-fa-v100_b200"), ROOT,
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", SCRIPT], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, "exit code %d\n%s\n%s" % (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    assert "side streams ok" in r.stdout
