"""Isolated quantized mul_mat on the B200 against the CPU oracle (BASELINE config 2's op sweep, every
shape, M up to 2048): single-stage programs through the C ABI, as the reference's
op tests run them (tests/unit/test_runtime_ops.py:86-102). The backend follows the oracle's reduction
order, so results are compared bit for bit."""

import numpy as np
import pytest

import oracle
from ggml_compiler_b200.programs import write_mul_mat
from ggml_compiler_b200.runtime import Model

pytestmark = pytest.mark.gpu


def weights(shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(0.02)


def run_mm(tmp_path, w, wtype, x):
    p = tmp_path / f"mm_{wtype}_{w.shape[0]}x{w.shape[1]}_{x.shape[0]}.gguf"
    write_mul_mat(p, w, wtype, x.shape[0])
    with Model(p) as m:
        return m.entries["main"](x=x[None])["out.0"].reshape(x.shape[0], w.shape[0])


# the three weight shapes at M = 1, 8, 64, 512 (and 2048 on the square one),
# plus small and ragged shapes (a row of 1000 tiles' worth, K not a multiple of the 128-block segment)
SWEEP = ([(4096, 4096, m) for m in (1, 8, 64, 512, 2048)] + [(14336, 4096, m) for m in (1, 8, 64, 512)] +
         [(4096, 14336, m) for m in (1, 8, 64, 512)] + [(256, 512, m) for m in (1, 8, 64)] +
         [(1000, 14336, m) for m in (1, 9, 64)])


@pytest.mark.parametrize("wtype", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K,M", SWEEP)
def test_quant_mul_mat_bit_exact(gpu, tmp_path, wtype, N, K, M):
    w = weights((N, K))
    x = np.random.default_rng(1).standard_normal((M, K), dtype=np.float32)
    got = run_mm(tmp_path, w, wtype, x)
    ref = oracle.mul_mat(oracle.quantize(w, wtype), wtype, K, x)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("wtype", ["f32", "f16"])
def test_float_mul_mat_bit_exact(gpu, tmp_path, wtype):
    w = weights((96, 160))
    x = np.random.default_rng(2).standard_normal((5, 160), dtype=np.float32)
    got = run_mm(tmp_path, w, wtype, x)
    wr = w.astype(np.float16) if wtype == "f16" else w
    np.testing.assert_array_equal(got, oracle.mul_mat(wr, wtype, 160, x))


def test_quant_mul_mat_edges(gpu, tmp_path):
    """Zero activation blocks (d = 0), huge and tiny values, a single block per row."""
    w = weights((64, 32))
    x = np.zeros((3, 32), np.float32)
    x[1, :5] = [1e4, -1e-30, 3.0, -3.0, 0.5]
    x[2] = np.linspace(-1, 1, 32, dtype=np.float32)
    for wtype in ("q4_0", "q8_0"):
        got = run_mm(tmp_path, w, wtype, x)
        np.testing.assert_array_equal(got, oracle.mul_mat(oracle.quantize(w, wtype), wtype, 32, x))


@pytest.mark.parametrize("wtype", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K,M", [(384, 1024, 9), (384, 1024, 64), (300, 2048, 200), (128, 256, 70)])
def test_quant_gemm_bit_exact(gpu, tmp_path, wtype, N, K, M):
    """9+ activation rows: the tensor-core GEMM (integer MMA per block, blocks summed in order),
    ragged in both the weight rows (N % 128) and the activation rows (M % 64)."""
    w = weights((N, K), seed=3)
    x = np.random.default_rng(4).standard_normal((M, K), dtype=np.float32)
    got = run_mm(tmp_path, w, wtype, x)
    ref = oracle.mul_mat(oracle.quantize(w, wtype), wtype, K, x)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("D,H,HKV,NQ,NKV,mask,kernel", [
    (128, 32, 8, 300, 700, "causal", "prefill"),  # GQA 4, 11 chunks, -65504 above the diagonal
    (128, 8, 8, 16, 130, "none", "prefill"),      # no GQA, no mask, ragged last chunk
    (64, 16, 2, 40, 260, "inf", "prefill"),       # GQA 8, -inf above the diagonal
    (64, 4, 4, 70, 64, "random", "prefill"),      # one chunk, finite random mask
    (128, 32, 8, 9, 700, "causal", "split"),      # fewer than 16 rows
    (128, 32, 8, 1, 768, "causal", "cluster"),    # one decode row: clusters of 12 chunks
    (64, 8, 2, 1, 130, "inf", "cluster"),         # one row, 3 chunks (ragged), hidden keys
    (128, 8, 8, 1, 1024, "none", "cluster"),      # one row, 16 chunks: the largest cluster
    (128, 32, 8, 1, 1100, "causal", "split"),     # one row, 18 chunks: the split kernel's global merge
])
def test_flash_attn_bit_exact(gpu, tmp_path, monkeypatch, D, H, HKV, NQ, NKV, mask, kernel):
    """flash_attn as a one-node program against the oracle, bit for bit, through the prefill kernel
    (16+ query rows), the split-KV kernel and the cluster kernel (one row, 2-16 chunks); the causal
    masks use the reference programs' -65504 (every chunk computed) or -inf (hidden chunks skipped by
    the merge), with rows whose keys are all hidden in the later chunks. The per-CTA trace shows
    which decode kernel ran: only the cluster kernel records its last stamp."""
    from ggml_compiler_b200.gguf_write import write_gguf
    from ggml_compiler_b200.programs import single_node_program
    from oracle.interp import Program

    rng = np.random.default_rng(D + H + NQ)
    q = rng.standard_normal((1, H, NQ, D), dtype=np.float32)
    k = (rng.standard_normal((1, HKV, NKV, D), dtype=np.float32) * 0.5).astype(np.float16)
    v = rng.standard_normal((1, HKV, NKV, D), dtype=np.float32).astype(np.float16)
    ins = [("q", "f32", [D, NQ, H, 1], [1, H, NQ, D]), ("k", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]),
           ("v", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D])]
    feed = {"q": q, "k": k, "v": v}
    if mask != "none":
        m = np.zeros((NQ, NKV), np.float32)
        if mask == "random":
            m = rng.standard_normal((NQ, NKV), dtype=np.float32) * 2
        else:
            hide = np.float32(-65504.0) if mask == "causal" else np.float32(-np.inf)
            for i in range(NQ):  # a decode row sees the first two thirds of the cache
                m[i, (NKV - NQ + i if NQ > 1 else 2 * NKV // 3) + 1:] = hide
        ins.append(("mask", "f16", [NKV, NQ, 1, 1], [1, 1, NQ, NKV]))
        feed["mask"] = m.astype(np.float16)[None, None]
    prog = single_node_program("flash_attn", ins, [n for n, *_ in ins], "f32", [D, H, NQ, 1], [1, NQ, H, D],
                               {"scale": float(1.0 / np.sqrt(D))})
    path = tmp_path / "fa.gguf"
    write_gguf(path, prog, [])
    trace = tmp_path / "trace.tsv"
    monkeypatch.setenv("GGML_COMPILER_B200_TRACE", str(trace))
    with Model(path) as m:
        got = m.entries["main"](**feed)["out.0"]
    want = Program(path).run("main", **feed)["out.0"]
    assert np.isfinite(got).all()
    np.testing.assert_array_equal(got, want)
    if kernel != "prefill":
        rows = [line.split("\t") for line in trace.read_text().splitlines() if "\tflash_attn\t" in line]
        assert rows, "no flash_attn stamps"
        cluster = {int(r[12]) >= 0 for r in rows}
        assert cluster == {kernel == "cluster"}, f"expected the {kernel} kernel"
