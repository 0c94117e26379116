"""ggml_compiler_b200_flash_attn_static (include/ggml_compiler_b200.h): split-KV flash attention on
caller-owned device buffers with the scratch in a static device array, so the call allocates
nothing. Checked through the C ABI against the existing path for the same op (a one-node flash_attn
program run by ggml_compiler_run, whose scratch lives in the call site's arena), on two calls in a
row with different inputs; the suite's tolerance for this kernel is exact equality. The file name
sorts last so the test also runs after every other test in one process; it passes alone too."""

import ctypes

import numpy as np
import pytest

from ggml_compiler_b200.gguf_write import write_gguf
from ggml_compiler_b200.programs import single_node_program
from ggml_compiler_b200.runtime import Model, load_library

D, H, HKV, NQ, NKV, CTX = 128, 8, 2, 3, 300, 512
SCALE = float(1.0 / np.sqrt(D))


def _entry(lib):
    f = lib.ggml_compiler_b200_flash_attn_static
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6 + [ctypes.c_float, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _inputs(seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((H, NQ, D), dtype=np.float32)
    cache_k = (rng.standard_normal((HKV, CTX, D), dtype=np.float32) * 0.5).astype(np.float16)
    cache_v = rng.standard_normal((HKV, CTX, D), dtype=np.float32).astype(np.float16)
    mask = (rng.standard_normal((NQ, NKV), dtype=np.float32) * 0.1).astype(np.float16)
    for i in range(NQ):  # causal tail: row i sees keys up to NKV - NQ + i
        mask[i, NKV - NQ + i + 1:] = -np.inf
    return q, cache_k, cache_v, mask


def _program_out(path, q, cache_k, cache_v, mask):
    """The op through the existing entry point: a one-node program, K/V as contiguous [Hkv, n_kv, D]."""
    with Model(path) as m:
        out = m.entries["main"](q=q[None], k=np.ascontiguousarray(cache_k[None, :, :NKV]),
                                v=np.ascontiguousarray(cache_v[None, :, :NKV]), mask=mask[None, None])["out.0"]
    return out.reshape(NQ, H, D)


@pytest.mark.gpu
def test_static_scratch_matches_program_path(gpu, tmp_path):
    import torch

    prog = single_node_program(
        "flash_attn",
        [("q", "f32", [D, NQ, H, 1], [1, H, NQ, D]), ("k", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]),
         ("v", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]), ("mask", "f16", [NKV, NQ, 1, 1], [1, 1, NQ, NKV])],
        ["q", "k", "v", "mask"], "f32", [D, H, NQ, 1], [1, NQ, H, D], {"scale": SCALE})
    path = tmp_path / "flash_attn.gguf"
    write_gguf(path, prog, [])
    f = _entry(load_library())
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    out = torch.empty((NQ, H, D), dtype=torch.float32, device=dev)
    for seed in (11, 12):  # two calls in a row through the static scratch
        q, ck, cv, mask = _inputs(seed)
        want = _program_out(path, q, ck, cv, mask)
        tq, tk, tv, tm = (torch.from_numpy(a).to(dev) for a in (q, ck, cv, mask))
        out.fill_(float("nan"))
        rc = f(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tm.data_ptr(), out.data_ptr(), D, NQ, H, NKV, HKV, CTX,
               SCALE, stream.cuda_stream)
        assert rc == 0, load_library().ggml_compiler_last_error().decode()
        stream.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_array_equal(got, want)


def test_static_scratch_rejects_oversized_calls(rtlib):
    """Sizes beyond the static scratch are refused on the host, before any device work (the pointers
    below are never dereferenced)."""
    f = _entry(rtlib)
    fake = 1 << 20  # 16-byte aligned, never touched: validation fails first
    # 64 query rows x 32 heads x 64 chunks of 130 floats: about 67 MiB of partials
    assert f(fake, fake, fake, fake, fake, 128, 64, 32, 4096, 8, 4096, 1.0, None) == -1
    msg = rtlib.ggml_compiler_last_error().decode()
    assert "static scratch holds 4.00 MiB" in msg, msg
    assert f(fake, fake, fake, None, fake, 96 + 8, 1, 8, 64, 8, 64, 1.0, None) == -1
    assert "multiple of 32" in rtlib.ggml_compiler_last_error().decode()
    assert f(fake, fake + 8, fake, None, fake, 128, 1, 8, 64, 8, 64, 1.0, None) == -1
    assert "16-byte aligned" in rtlib.ggml_compiler_last_error().decode()
    assert f(fake, fake, fake, None, fake, 128, 1, 8, 64, 8, 32, 1.0, None) == -1
    assert "kv_head_stride" in rtlib.ggml_compiler_last_error().decode()
