"""ggml_compiler_b200_flash_attn_static (include/ggml_compiler_b200.h): flash attention on
caller-owned device buffers with the scratch in a static device array, so the call allocates
nothing. Some callers cannot let a library allocate: a custom op inside another engine's decode
loop, whose caching allocator already holds the free device memory (cudaMalloc may fail) and whose
other streams a cudaMalloc / cudaFree would stall by synchronising the device.

Checked through the C ABI on two calls in a row with different inputs, for two GQA shapes (3 query
rows: the per-chunk kernel and the static partials; 24 rows: the kernel that merges inside each CTA),
against the existing path for the same op (a one-node flash_attn program, whose scratch lives in the
call site's arena) and against the CPU oracle; this suite's tolerance for the kernel is exact
equality. Around the second call the device's free memory stays the same. The file name sorts last
so the test also runs after every other test in one process; it passes alone too."""

import ctypes

import numpy as np
import pytest

from ggml_compiler_b200.gguf_write import write_gguf
from ggml_compiler_b200.programs import single_node_program
from ggml_compiler_b200.runtime import Model, load_library
from oracle.interp import Program

D, H, HKV, NKV, CTX = 128, 8, 2, 300, 512
SCALE = float(1.0 / np.sqrt(D))


def _entry(lib):
    f = lib.ggml_compiler_b200_flash_attn_static
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6 + [ctypes.c_float, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _inputs(seed, nq):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((H, nq, D), dtype=np.float32)
    cache_k = (rng.standard_normal((HKV, CTX, D), dtype=np.float32) * 0.5).astype(np.float16)
    cache_v = rng.standard_normal((HKV, CTX, D), dtype=np.float32).astype(np.float16)
    mask = (rng.standard_normal((nq, NKV), dtype=np.float32) * 0.1).astype(np.float16)
    for i in range(nq):  # causal tail: row i sees keys up to NKV - nq + i
        mask[i, NKV - nq + i + 1:] = -np.inf
    return q, cache_k, cache_v, mask


def _feed(q, cache_k, cache_v, mask):
    """The program's inputs: K/V as contiguous [Hkv, n_kv, D] (the static call reads the cache rows)."""
    return {"q": q[None], "k": np.ascontiguousarray(cache_k[None, :, :NKV]),
            "v": np.ascontiguousarray(cache_v[None, :, :NKV]), "mask": mask[None, None]}


@pytest.mark.gpu
@pytest.mark.parametrize("nq", [3, 24])
def test_static_scratch_matches_program_path_and_oracle(gpu, tmp_path, nq):
    import torch

    prog = single_node_program(
        "flash_attn",
        [("q", "f32", [D, nq, H, 1], [1, H, nq, D]), ("k", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]),
         ("v", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]), ("mask", "f16", [NKV, nq, 1, 1], [1, 1, nq, NKV])],
        ["q", "k", "v", "mask"], "f32", [D, H, nq, 1], [1, nq, H, D], {"scale": SCALE})
    path = tmp_path / "flash_attn.gguf"
    write_gguf(path, prog, [])
    f = _entry(load_library())
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    out = torch.empty((nq, H, D), dtype=torch.float32, device=dev)
    for call, seed in enumerate((11, 12)):  # two calls in a row through the static scratch
        q, ck, cv, mask = _inputs(seed, nq)
        with Model(path) as m:
            want = m.entries["main"](**_feed(q, ck, cv, mask))["out.0"].reshape(nq, H, D)
        oracle_out = Program(path).run("main", **_feed(q, ck, cv, mask))["out.0"].reshape(nq, H, D)
        tq, tk, tv, tm = (torch.from_numpy(a).to(dev) for a in (q, ck, cv, mask))
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = f(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tm.data_ptr(), out.data_ptr(), D, nq, H, NKV, HKV, CTX,
               SCALE, stream.cuda_stream)
        assert rc == 0, load_library().ggml_compiler_last_error().decode()
        stream.synchronize()
        if call == 1:  # the set-up is done: the call itself takes no device memory
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(got, oracle_out)


def test_static_scratch_rejects_oversized_calls(rtlib):
    """Sizes beyond the static scratch are refused on the host, before any device work (the pointers
    below are never dereferenced)."""
    f = _entry(rtlib)
    fake = 1 << 20  # 16-byte aligned, never touched: validation fails first
    # 8 query rows (the per-chunk kernel) x 32 heads x 1024 chunks of 130 floats: about 136 MiB
    assert f(fake, fake, fake, fake, fake, 128, 8, 32, 65536, 8, 65536, 1.0, None) == -1
    msg = rtlib.ggml_compiler_last_error().decode()
    assert "static scratch holds 4.00 MiB" in msg, msg
    assert f(fake, fake, fake, None, fake, 96 + 8, 1, 8, 64, 8, 64, 1.0, None) == -1
    assert "multiple of 32" in rtlib.ggml_compiler_last_error().decode()
    assert f(fake, fake + 8, fake, None, fake, 128, 1, 8, 64, 8, 64, 1.0, None) == -1
    assert "16-byte aligned" in rtlib.ggml_compiler_last_error().decode()
    assert f(fake, fake, fake, None, fake, 128, 1, 8, 64, 8, 32, 1.0, None) == -1
    assert "kv_head_stride" in rtlib.ggml_compiler_last_error().decode()
