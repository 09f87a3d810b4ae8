"""Stream ordering with programmatic dependent launch.

The forward and backward kernels are launched so that they may start their set-up
while the kernel before them on the stream is still running; each waits for that
kernel to complete before it touches global memory.  These tests feed every kernel
inputs that the kernel right before it on the same stream has just written -- a
torch elementwise kernel, or the library's own previous call -- and require results
bitwise equal to the same calls separated by a device synchronisation (the kernels
are deterministic, so any read of stale data would show)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

B, H, S, D = 2, 4, 640, 128


@pytest.fixture(scope="module")
def api():
    import co_alibi_attn
    return co_alibi_attn


def _inputs(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g).to(torch.float16).cuda() for _ in range(4)]


def test_forward_reads_what_the_previous_kernel_wrote(api):
    q0, k0, v0, _ = _inputs(11)

    def run(sync):
        # each operand comes out of a torch kernel launched immediately before the call
        q = q0 * 1.5
        k = k0 - 0.25
        v = v0 * 0.5
        if sync:
            torch.cuda.synchronize()
        return api.co_alibi_attention(q, k, v, causal=True)

    ref = run(True)
    torch.cuda.synchronize()
    for _ in range(3):
        assert torch.equal(run(False), ref)
    assert api.device_status(reset=True) == 0


def test_chained_calls_read_the_previous_call_outputs(api):
    q, k, v, do = _inputs(12)

    def run(sync):
        qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
        o1 = api.co_alibi_attention(qs, ks, vs, causal=True)
        if sync:
            torch.cuda.synchronize()
        o2 = api.co_alibi_attention(o1, ks, vs, causal=True)   # the forward reads o1 right after it is written
        if sync:
            torch.cuda.synchronize()
        o2.backward(do)                                       # backward kernels back to back on one stream
        if sync:
            torch.cuda.synchronize()
        return o2.detach(), qs.grad, ks.grad, vs.grad

    ref = run(True)
    torch.cuda.synchronize()
    for _ in range(2):
        got = run(False)
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert api.device_status(reset=True) == 0


def test_torch_kernel_after_the_backward_sees_finished_gradients(api):
    q, k, v, do = _inputs(13)
    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    api.co_alibi_attention(qs, ks, vs, causal=False).backward(do)
    early = torch.cat([ks.grad.float().sum(dim=-1), vs.grad.float().sum(dim=-1)])  # right after the last kernel
    torch.cuda.synchronize()
    late = torch.cat([ks.grad.float().sum(dim=-1), vs.grad.float().sum(dim=-1)])
    assert torch.equal(early, late)
    assert api.device_status(reset=True) == 0
