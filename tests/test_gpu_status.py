"""Device-side timeouts reach the caller as an exception (the reference's TORCH_CHECK failures
surface as RuntimeError, kernels/hip/rmsnorm.py:119-123).

The failure is made without faulting or hanging the GPU: the library's probe kernel waits on an
mbarrier that nothing completes, with a limit of 1000 polls, so its bounded wait runs out, writes
AK_ERR_TIMEOUT to the caller's status word and returns."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_bounded_wait_timeout_raises_and_context_stays_usable():
    from kernels import _ak
    with pytest.raises(_ak.AkError, match="bounded device-side wait gave up"):
        _ak.test_bounded_wait(DEV, max_spins=1000)
    # reported once, then cleared
    _ak.check_status(DEV)
    # the context still runs kernels
    x = torch.randn(64, 256, device=DEV)
    y = _ak.softmax_fwd(x)
    torch.testing.assert_close(y, torch.softmax(x, -1), rtol=1e-5, atol=1e-6)


def test_timeout_of_an_earlier_call_raises_on_the_next_call_of_its_family():
    """Without a sync, the failure is raised by the next call that uses the same status word."""
    from kernels import _ak
    _ak.call("ak_test_bounded_wait", _ak.status_ptr(DEV, "bounded_wait_test"), 1000, _ak.stream(DEV))
    torch.cuda.synchronize(DEV)
    with pytest.raises(_ak.AkError, match="bounded_wait_test"):
        _ak.status_ptr(DEV, "bounded_wait_test")
    _ak.check_status(DEV)


def test_probe_rejects_bad_limits():
    from kernels import _ak
    with pytest.raises(_ak.AkError, match="max_spins"):
        _ak.call("ak_test_bounded_wait", _ak.status_ptr(DEV, "bounded_wait_test"), 0, _ak.stream(DEV))


def test_normal_calls_leave_the_status_clear():
    from kernels import _ak
    g = torch.Generator().manual_seed(0)
    b, dim, L, N = 2, 16, 600, 16
    u = torch.randn(b, dim, L, generator=g).to(torch.bfloat16).to(DEV)
    delta = (torch.randn(b, dim, L, generator=g) - 4.6).to(torch.bfloat16).to(DEV)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(dim, 1).to(DEV)
    Bm = torch.randn(b, N, L, generator=g).to(torch.bfloat16).to(DEV)
    Cm = torch.randn(b, N, L, generator=g).to(torch.bfloat16).to(DEV)
    out, last, states = _ak.selective_scan_fwd(u, delta, A, Bm, Cm, None, None, None, True)
    _ak.selective_scan_bwd(torch.ones_like(out), u, delta, A, Bm, Cm, None, None, None, True, states)
    H = torch.randn(256, 64, device=DEV).to(torch.bfloat16)
    W = torch.randn(512, 64, device=DEV).to(torch.bfloat16)
    lab = torch.randint(0, 512, (256,), device=DEV)
    _ak.linear_ce_fwdbwd(H, W, lab)
    _ak.check_status(DEV)


def test_status_words_set_up_in_a_fresh_process():
    """The first library call of a process may be one that needs a status word (it is created
    under the same lock that loads the library)."""
    import subprocess
    import sys
    code = ("import sys; sys.path[:0] = ['autokernel-halo-strix_b200', '.']\n"
            "import torch\nfrom kernels import _ak\n"
            "a = torch.randn(256, 64, device='cuda').to(torch.bfloat16)\n"
            "c = _ak.tc_gemm(a, a.t())\n_ak.check_status()\nprint('ok')\n")
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    out = subprocess.run([sys.executable, "-c", code], cwd=repo, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]
