"""C ABI checks that need no GPU: libcbx_ops.so loads, exports every symbol
include/cbx_ops.h declares, rejects bad arguments on the host (before any CUDA
call), and its host-side table builders match the oracle.  CPU only."""
import ctypes
import os
import re
import subprocess
import threading

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cbx_ops.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"CBX_API\s+[\w\s\*]+?\b(cbx_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from chatterbox_amdvulkan_b200 import _lib, build
    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.load()


def test_header_declares_the_planned_entry_points():
    names = _declared()
    for n in ("cbx_embed_gather_add", "cbx_add_layernorm", "cbx_layernorm_channels",
              "cbx_gelu_tanh", "cbx_silu", "cbx_mish", "cbx_timestep_embed",
              "cbx_sinusoid_freqs", "cbx_snake", "cbx_snake_alpha_inv", "cbx_last_error",
              "cbx_version", "cbx_status_string", "cbx_gelu_erf", "cbx_bias_act",
              "cbx_sum3_scale", "cbx_device_errors", "cbx_nsf_source", "cbx_stft",
              "cbx_istft_post", "cbx_hann_window", "cbx_embed_gather_add_batched",
              "cbx_t3_embed_sequence_batched"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from chatterbox_amdvulkan_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(cbx_\w+)$", out, re.M))
    declared = set(_declared())
    assert declared <= exported, declared - exported
    # nothing else leaks out of the library under the cbx_ prefix
    assert exported == declared, exported - declared
    # and the ctypes table covers exactly the header
    assert set(_lib.SIGNATURES) == declared


def test_version_and_status_strings(lib):
    assert lib.cbx_version() == 0x000100
    assert lib.cbx_status_string(0) == b"CBX_OK"
    assert lib.cbx_status_string(-1) == b"CBX_ERR_INVALID_ARG"
    assert lib.cbx_status_string(-5) == b"CBX_ERR_TIMEOUT"


FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: every call below fails validation


@pytest.mark.parametrize("call,status,msg", [
    (lambda L: L.cbx_gelu_tanh(None, None, 16, 0, None), -1, "NULL"),
    (lambda L: L.cbx_silu(FAKE, FAKE, -1, 0, None), -1, "< 0"),
    (lambda L: L.cbx_mish(FAKE, FAKE, 16, 7, None), -2, "unsupported type"),
    (lambda L: L.cbx_add_layernorm(FAKE, None, 0, 0, None, None, 1e-5, 4, 0, None, FAKE, 0, 0,
                                   None), -1, "hidden"),
    (lambda L: L.cbx_add_layernorm(FAKE, None, 5, 0, None, None, 1e-5, 4, 8, None, FAKE, 0, 0,
                                   None), -2, "in_type"),
    (lambda L: L.cbx_add_layernorm(FAKE, None, 0, 4, None, None, 1e-5, 4, 8, None, FAKE, 0, 0,
                                   None), -1, "stride"),
    (lambda L: L.cbx_add_layernorm(FAKE, None, 0, 0, None, None, -1.0, 4, 8, None, FAKE, 0, 0,
                                   None), -1, "eps"),
    (lambda L: L.cbx_layernorm_channels(FAKE, None, None, 1e-5, None, 1, 4, 4, 3, 1, FAKE,
                                        None), -1, "layout"),
    (lambda L: L.cbx_layernorm_channels(FAKE, None, None, 1e-5, None, 1, 4, 4, 0, 9, FAKE,
                                        None), -1, "act"),
    (lambda L: L.cbx_causal_block1d_tail(FAKE, None, None, None, 1e-5, None, 1, 4, 4, 9, FAKE,
                                         None), -1, "act"),
    (lambda L: L.cbx_causal_block1d_tail(FAKE, None, None, None, 1e-5, None, 1, 4, 4, 1, FAKE,
                                         None), -1, "alias"),
    (lambda L: L.cbx_causal_block1d_tail(FAKE, None, None, None, 1e-5, None, 1, 0, 4, 1,
                                         ctypes.c_void_p(0x2000), None), -1, "C 0"),
    (lambda L: L.cbx_timestep_embed(FAKE, 4, FAKE, 2, 1000.0, 0, FAKE, None), -1, "dim"),
    (lambda L: L.cbx_timestep_embed(FAKE, 4, FAKE, 320, 1000.0, 1, FAKE, None), -1, "act"),
    (lambda L: L.cbx_snake(FAKE, None, None, 1e-9, 1, 4, 4, 0, FAKE, None), -1, "NULL"),
    (lambda L: L.cbx_snake(FAKE, FAKE, None, 1e-9, 1, 0, 4, 0, FAKE, None), -1, "C 0"),
    (lambda L: L.cbx_embed_gather_add(FAKE, 3, 10, None, 0, 0, FAKE, None, 0, 4, 8, FAKE, 0,
                                      None, None), -2, "types"),
    (lambda L: L.cbx_embed_gather_add(None, 0, 10, None, 0, 0, FAKE, None, 0, 4, 8, FAKE, 0,
                                      None, None), -1, "NULL"),
    (lambda L: L.cbx_embed_gather_add_batched(FAKE, 0, 10, FAKE, 0, 10, FAKE, 2, 3, -1, 8,
                                              FAKE, 0, None, None), -1, "n_past"),
    (lambda L: L.cbx_embed_gather_add_batched(FAKE, 0, 10, FAKE, 9, 10, FAKE, 2, 3, 0, 8,
                                              FAKE, 0, None, None), -2, "types"),
    (lambda L: L.cbx_embed_gather_add_batched(FAKE, 0, 10, None, 0, 0, None, 2, 3, 0, 8,
                                              FAKE, 0, None, None), -1, "NULL"),
    (lambda L: L.cbx_embed_gather_add_batched(FAKE, 0, 10, None, 0, 0, FAKE, 1 << 40, 1 << 20,
                                              0, 1024, FAKE, 0, None, None), -1, "overflows"),
    (lambda L: L.cbx_t3_embed_sequence_batched(None, 0, None, 1, 0, None, 0, FAKE, 1, 10, FAKE,
                                               4, FAKE, 1, 10, 0, 8, -2, FAKE, 0, None, None),
     -1, "n_batch"),
    (lambda L: L.cbx_t3_embed_sequence_batched(None, 1, None, 1, 0, None, 0, FAKE, 1, 10, FAKE,
                                               4, FAKE, 1, 10, 0, 8, 3, FAKE, 0, None, None),
     -1, "NULL"),
    (lambda L: L.cbx_t3_embed_sequence_batched(None, 0, None, 1, 0, None, 0, FAKE, 1, 10, FAKE,
                                               1 << 20, FAKE, 1, 10, 0, 1 << 20, 1 << 30, FAKE, 0,
                                               None, None), -1, "overflows"),
    (lambda L: L.cbx_bias_act(FAKE, FAKE, 0, 4, 8, FAKE, 0, 7, 3, 0.0, None), -1, "bias_len"),
    (lambda L: L.cbx_bias_act(FAKE, FAKE, 0, 4, 8, None, 2, 0, 3, 0.0, None), -1, "bias_axis"),
    (lambda L: L.cbx_bias_act(FAKE, FAKE, 0, 4, 8, None, 0, 0, 7, 0.0, None), -1, "act"),
    (lambda L: L.cbx_bias_act(FAKE, FAKE, 5, 4, 8, None, 0, 0, 3, 0.0, None), -2, "type"),
    (lambda L: L.cbx_sum3_scale(FAKE, None, FAKE, 0.5, FAKE, 16, 0, None), -1, "NULL"),
    (lambda L: L.cbx_gelu_erf(FAKE, FAKE, 16, 9, None), -2, "unsupported type"),
    (lambda L: L.cbx_nsf_source(FAKE, 2, 10, 0, 24000, FAKE, FAKE, FAKE, 0.0, FAKE, None), -1,
     "upsample"),
    (lambda L: L.cbx_nsf_source(FAKE, 2, 10, 480, 24000, None, FAKE, FAKE, 0.0, FAKE, None), -1,
     "NULL"),
    (lambda L: L.cbx_stft(FAKE, 1, 100, 15, 4, FAKE, 1, FAKE, None), -1, "n_fft"),
    (lambda L: L.cbx_stft(FAKE, 1, 8, 16, 4, FAKE, 1, FAKE, None), -1, "reflect"),
    (lambda L: L.cbx_stft(FAKE, 1, 100, 16, 4, FAKE, 5, FAKE, None), -1, "layout"),
    (lambda L: L.cbx_istft_post(FAKE, 1, 10, 16, 0, FAKE, 1, 0.99, FAKE, None), -1, "hop"),
    (lambda L: L.cbx_istft_post(FAKE, 1, 10, 16, 4, FAKE, 1, -1.0, FAKE, None), -1,
     "audio_limit"),
    (lambda L: L.cbx_hann_window(0, None), -1, "bad arguments"),
    (lambda L: L.cbx_qkv_kv_append(FAKE, 0, None, 2, 8, FAKE, 0, FAKE, FAKE, 0, 8, 4, None, FAKE,
                                   None), -1, "overlap"),
    (lambda L: L.cbx_t3_embed_sequence(None, 1, None, 1, 0, None, 0, FAKE, 1, 10, FAKE, 4, FAKE,
                                       1, 10, 0, 8, FAKE, 0, None, None), -1, "NULL"),
    (lambda L: L.cbx_t3_embed_sequence(None, 0, None, 1, 0, None, 0, FAKE, 7, 10, FAKE, 4, FAKE,
                                       1, 10, 0, 8, FAKE, 0, None, None), -2, "types"),
    (lambda L: L.cbx_t3_embed_sequence(None, 0, None, 1, 0, None, 0, FAKE, 1, 10, FAKE, 4, FAKE,
                                       1, 10, -3, 8, FAKE, 0, None, None), -1, "n_past"),
])
def test_host_validation_rejects_before_launch(lib, call, status, msg):
    assert call(lib) == status
    assert msg in lib.cbx_last_error().decode()


def test_zero_sized_calls_succeed_without_a_device(lib):
    assert lib.cbx_gelu_tanh(None, None, 0, 0, None) == 0
    assert lib.cbx_last_error() == b""
    assert lib.cbx_snake(None, None, None, 1e-9, 0, 4, 4, 0, None, None) == 0


def test_host_sinusoid_freqs_match_oracle(lib):
    from chatterbox_amdvulkan_b200 import ops
    for dim in (4, 9, 64, 320, 1024):
        assert np.array_equal(ops.sinusoid_freqs(dim), O.sinusoid_freqs(dim))
    out = np.empty(4, np.float32)
    assert lib.cbx_sinusoid_freqs(3, out.ctypes.data_as(ctypes.c_void_p)) == -1


def test_host_hann_window_matches_oracle(lib):
    from chatterbox_amdvulkan_b200 import ops
    for n in (4, 16, 20, 32):
        assert np.array_equal(ops.hann_window(n), O.hann_window(n))


def test_host_snake_alpha_inv_matches_engine_expression(lib):
    from chatterbox_amdvulkan_b200 import ops
    rng = np.random.default_rng(0)
    a = np.exp(0.3 * rng.standard_normal(512)).astype(np.float32)
    inv = ops.snake_alpha_inv(a)
    assert np.array_equal(inv, O.snake_alpha_inv(a))
    assert np.array_equal(inv, (np.float32(1.0) / (a + np.float32(1e-9))).astype(np.float32))


def test_ops_refuse_cpu_tensors(lib):
    torch = pytest.importorskip("torch")
    from chatterbox_amdvulkan_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.gelu(torch.zeros(8))
    with pytest.raises(ValueError, match="CUDA"):
        ops.snake(torch.zeros(1, 4, 4), torch.ones(4))


def _kv_args(torch, n_rows=4, D=8, ctx=6, slab=None, cache_elems=None, n_pos=None):
    slab = ctx * D if slab is None else slab
    need = (n_rows - 1) * slab + ctx * D
    n = need if cache_elems is None else cache_elems
    return dict(qkv=torch.zeros(n_rows, 3 * D), bias=torch.zeros(3 * D),
                cache_k=torch.zeros(n), cache_v=torch.zeros(n),
                positions=torch.zeros(n_rows if n_pos is None else n_pos, dtype=torch.int32),
                slab_stride=slab, max_context=ctx)


@pytest.mark.parametrize("kw,msg", [
    (dict(cache_elems=4 * 6 * 8 - 1), "need"),          # last slab one element short
    (dict(slab=5 * 8), "overlap"),                      # slabs overlap
    (dict(n_pos=3), "positions"),                       # fewer positions than rows
])
def test_qkv_kv_append_wrapper_checks_sizes_before_launch(kw, msg):
    """The torch wrapper has the tensors' sizes (the C ABI only pointers): it
    refuses caches too small for the rows' slabs, overlapping slabs and short
    position lists before anything reaches the device."""
    torch = pytest.importorskip("torch")
    from chatterbox_amdvulkan_b200 import ops
    with pytest.raises(ValueError, match=msg):
        ops.qkv_kv_append(**_kv_args(torch, **kw))
    a = _kv_args(torch, **kw)
    a["qkv"] = torch.zeros(4, 25)
    with pytest.raises(ValueError, match="multiple of 3"):
        ops.qkv_kv_append(**a)
    a = _kv_args(torch)            # sizes fine: only then the CPU tensor is refused
    with pytest.raises(ValueError, match="CUDA"):
        ops.qkv_kv_append(**a)


def test_product_package_never_touches_the_oracle():
    pkg = os.path.join(ROOT, "chatterbox_amdvulkan_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                src = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(import|from)\s+oracle\b", src, re.M), f
                assert "cbx_oracle" not in src and "libcbx_oracle" not in src, f


def test_last_error_is_thread_local(lib):
    L = lib
    ready = threading.Barrier(2)
    seen = {}

    def bad(tag, call, key):
        ready.wait()
        for _ in range(200):
            rc = call()
            msg = L.cbx_last_error().decode()
            if key not in msg or rc >= 0:
                seen[tag] = (rc, msg)
                return
        seen[tag] = "ok"

    fake = ctypes.c_void_p(0x1000)
    t1 = threading.Thread(target=bad, args=(
        "snake", lambda: L.cbx_snake(fake, None, None, 1e-9, 1, 4, 4, 0, fake, None), "cbx_snake"))
    t2 = threading.Thread(target=bad, args=(
        "gelu", lambda: L.cbx_gelu_tanh(fake, fake, 16, 7, None), "cbx_gelu_tanh"))
    t1.start()
    t2.start()
    t1.join(timeout=60)
    t2.join(timeout=60)
    assert seen == {"snake": "ok", "gelu": "ok"}, seen
