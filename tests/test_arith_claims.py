"""CPU checks of the arithmetic identities the GPU kernels rely on to stay bit-identical with the
CPU checker (no GPU needed; numpy float32 stands in for the device's IEEE single operations).

- The tensor-core GEMM's epilogue turns an int32 block sum into a float through the 1.5 * 2^23
  bias (bits 0x4B400000 + isum, minus 12582912.0f). This is exact for every |isum| < 2^22; a Q8_0
  or Q4_0 block sum is at most 32 * 127 * 127 (the activation codes are within ±127, the weight
  codes within ±128 at the extreme).
- The flash-prefill kernel combines a head dot's 32 lane chains pairwise in bit-reversed lane
  order. That equals the value every lane holds after the xor butterfly the split-KV kernel and
  the checker use (off = 16, 8, 4, 2, 1).
- The flash-prefill kernel skips a chunk in its first pass when |q|_1 · max|k| · |scale| (× 1.01,
  + 1) plus the chunk's largest mask value lies 128 below a maximum already seen. The bound must
  hold for the float32 dot as computed: lane chains of fmas, then the tree.
- Batched decode attends over one window per step with a -inf mask past each sequence's position;
  the checker's attention gives the same bits over any window and either mask value."""

import numpy as np

f32 = np.float32


def test_biased_int_to_float_is_exact():
    isum = np.arange(-(1 << 22), 1 << 22, dtype=np.int64)
    bits = (np.int64(0x4B400000) + isum).astype(np.uint32)
    via_bias = bits.view(np.float32) - f32(12582912.0)
    np.testing.assert_array_equal(via_bias, isum.astype(np.float32))
    assert 32 * 127 * 128 < (1 << 22)


def _butterfly(p):
    """Lane values after the xor butterfly (every lane adds its partner's value)."""
    v = p.copy()
    for off in (16, 8, 4, 2, 1):
        v = (v + v[np.arange(32) ^ off]).astype(np.float32)
    return v


def _pairwise_bitrev(p):
    """The prefill kernel's order: leaves in bit-reversed lane order, combined like a binary counter."""
    stack = [None] * 6
    for i in range(32):
        lane = int(f"{i:05b}"[::-1], 2)
        v = p[lane]
        lv = 0
        while (i >> lv) & 1:
            v = f32(stack[lv] + v)
            lv += 1
        stack[lv] = v
    return stack[5]


def test_bitreversed_pairwise_equals_butterfly():
    rng = np.random.default_rng(0)
    for scale in (1e-3, 1.0, 1e3, 1e30):
        for _ in range(200):
            p = (rng.standard_normal(32) * scale).astype(np.float32)
            b = _butterfly(p)
            assert np.all(b == b[0]), "every lane holds the same value"
            assert _pairwise_bitrev(p) == b[0]


def _lane_chain_dot(q, k):
    """The checker's head dot: lane l runs an fma chain over elements [l*D/32, (l+1)*D/32)."""
    D = q.shape[0]
    c = D // 32
    p = np.zeros(32, np.float32)
    for l in range(32):
        acc = f32(0.0)
        for j in range(c):
            acc = f32(np.float64(q[l * c + j]) * np.float64(k[l * c + j]) + np.float64(acc))  # fma, emulated (exact f16 products)
        p[l] = acc
    return _butterfly(p)[0]


def test_score_bound_holds():
    rng = np.random.default_rng(1)
    for D in (64, 128):
        for scale_q in (0.1, 1.0, 30.0):
            for _ in range(100):
                q = (rng.standard_normal(D) * scale_q).astype(np.float16).astype(np.float32)
                k = (rng.standard_normal(D) * rng.uniform(0.1, 20)).astype(np.float16).astype(np.float32)
                scale = f32(1.0 / np.sqrt(D))
                s = abs(f32(_lane_chain_dot(q, k) * scale))
                l1 = f32(0.0)
                for x in q:
                    l1 = f32(l1 + abs(x))
                bound = f32(f32(f32(f32(l1 * np.max(np.abs(k))) * scale) * f32(1.01)) + f32(1.0))
                assert s <= bound


def test_attention_window_past_the_position_changes_nothing():
    """Batched decode attends each sequence over one window for the whole step (the longest
    sequence's, in 256-key steps) with a -inf mask past the sequence's position; the single-sequence
    decode attends over its own window with the reference programs' -65504 mask. The checker's
    64-key chunks merged in order give the same bits either way: a key past the position weighs
    exactly 0, and a chunk wholly past it adds exactly 0 to the merge."""
    import ctypes

    import oracle

    lib = oracle.lib()
    rng = np.random.default_rng(5)
    D, pos = 128, 300
    q = rng.standard_normal(D, dtype=np.float32)
    k = (rng.standard_normal((2304, D), dtype=np.float32) * 0.5).astype(np.float16)
    v = rng.standard_normal((2304, D), dtype=np.float32).astype(np.float16)
    q = q.astype(np.float16).astype(np.float32)  # the kernels round the query to f16 first

    def row(nkv, hide):
        m = np.zeros(nkv, np.float32)
        m[pos + 1:] = hide
        mh = np.ascontiguousarray(m.astype(np.float16)).view(np.uint16)
        kk = np.ascontiguousarray(k[:nkv]).view(np.uint16)
        vv = np.ascontiguousarray(v[:nkv]).view(np.uint16)
        out = np.empty(D, np.float32)
        lib.orc_flash_attn_row(q.ctypes.data, kk.ctypes.data, D, vv.ctypes.data, D, nkv, D, mh.ctypes.data,
                               ctypes.c_float(1.0 / np.sqrt(D)), out.ctypes.data)
        return out

    want = row(768, -65504.0)  # the decode entry: n_kv 768, the reference's clamped mask
    for nkv in (320, 512, 1024, 2304):
        np.testing.assert_array_equal(row(nkv, -np.inf), want)
        np.testing.assert_array_equal(row(nkv, -65504.0), want)
