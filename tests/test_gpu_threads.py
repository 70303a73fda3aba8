"""libcbx_ops is reentrant and thread-safe across streams: host threads, each
on its own CUDA stream, call the same entry points at the same time, and every
result equals the single-threaded one bit for bit (the thread-local error
message is checked on the CPU in test_abi.py)."""
import threading

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import _lib, ops
    return ops, _lib.load()


def _work(ops, x, r, g, b, xc, gc, bc, alpha):
    y, s = ops.add_layernorm(x, r, g, b, 1e-5, return_sum=True)
    u = ops.gelu(y)
    c = ops.layernorm_channels(xc, gc, bc, 1e-5, None, layout="BCT", act="mish")
    z = ops.snake(xc, alpha)
    return [y, s, u, c, z]


def test_concurrent_streams_match_serial(env):
    ops, _ = env
    gen = torch.Generator(device="cuda").manual_seed(0)
    n_threads, iters = 6, 20
    inputs = []
    for _ in range(n_threads):
        x = torch.randn(300, 1024, generator=gen, device="cuda")
        r = torch.randn(300, 1024, generator=gen, device="cuda")
        g = 1 + 0.1 * torch.randn(1024, generator=gen, device="cuda")
        b = 0.1 * torch.randn(1024, generator=gen, device="cuda")
        xc = torch.randn(2, 256, 200, generator=gen, device="cuda")
        gc = 1 + 0.1 * torch.randn(256, generator=gen, device="cuda")
        bc = 0.1 * torch.randn(256, generator=gen, device="cuda")
        alpha = torch.exp(0.3 * torch.randn(256, generator=gen, device="cuda"))
        inputs.append((x, r, g, b, xc, gc, bc, alpha))
    serial = [[t.clone() for t in _work(ops, *inp)] for inp in inputs]
    torch.cuda.synchronize()
    results = [None] * n_threads
    errors = []
    barrier = threading.Barrier(n_threads)

    def run(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                barrier.wait()
                for _ in range(iters):
                    out = _work(ops, *inputs[i])
                s.synchronize()
                results[i] = out
        except Exception as e:  # surfaced below
            errors.append(e)

    th = [threading.Thread(target=run, args=(i,)) for i in range(n_threads)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    assert not errors, errors
    for i in range(n_threads):
        for a, b in zip(results[i], serial[i]):
            assert torch.equal(a, b)
