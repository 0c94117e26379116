"""Benchmark: 8B-shape Q4_0 batch-1 decode on the B200 backend.

A Llama-3-8B-shaped model (32 layers, d_model 4096, 32/8 heads, head 128, FFN 14336, vocab 128256,
RoPE theta 500000) with N(0, 0.02) weights from seed 0, projections and output head in Q4_0, is
written as a ggml-compiler GGUF (the program the reference compiler emits for that shape at -O3)
and loaded through the C ABI. A 512-token prompt (seed 1) is prefilled, then greedy decode steps
are timed (one step = one token through all 32 layers; n_kv = 768).

- value: decode tok/s with every input resident on the device: the program's `generate` entry
  runs K steps back to back (device loop); time from CUDA events on the model's stream.
- e2e: the same decode through the public C API from host buffers, one `decode` entry per token
  (host -> device copies of token/position/mask from pinned memory, device -> host logits, host
  argmax), timed with CUDA events on the same stream.
- roofline: the weight-streaming kernels (the fused GEMV launches), algorithmic bytes per launch
  (Q4_0 weight bytes + activation bytes) / mean launch time from a profiled pass of the same steps
  (each launch timed with CUDA events on the model's stream); `step_hbm_frac` is the same weight
  bytes over the timed step itself.
- cpu_baseline / --impl reference: the reference's CPU arithmetic (this repository's C
  restatement of ggml's CPU path, oracle/) timed on the host's cores on decode steps of the same
  model at the same n_kv. The reference arm loads no product code.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 8b|tiny|sweep]
    python bench.py --config sweep [--shape NxK] [--m M] [--wtype q4_0|q8_0]   # config 2, one line per case
    python bench.py --config prefill   # config 4: 8 x 2048-token Q8_0 prefill, tensor-core roofline
    python bench.py --config attn      # isolated flash_attn at the 8B shape (prefill and decode rows)
    python bench.py --config 70b [--gpus N --parallel tp]   # config 5 shape, tensor parallel over N GPUs
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "ggml-compiler_b200"))
sys.path.insert(0, str(REPO))

METRIC = "8B-shape Q4_0 decode tok/s; quant-GEMV HBM GB/s as % of B200 peak"
# DRAM traffic / algorithmic bytes from ncu captures of the same kernels: the GEMV moves
# 9,515,264 B for 9,469,952 algorithmic; the GEMM 11,694,336 B for 11,665,408 (weights + codes + scales)
GEMV_TRAFFIC_RATIO = 9515264 / 9469952
GEMM_TRAFFIC_RATIO = 11694336 / 11665408
CACHE = Path(os.environ.get("GCB_BENCH_CACHE", "/tmp/gcb_bench"))


def shape_for(config: str):
    """(shape, workload, prompt tokens, n_kv of the timed decode steps)."""
    from ggml_compiler_b200.llm import LLAMA3_8B, LLAMA3_70B, TINY, LlamaShape

    if config == "8b":
        return LLAMA3_8B, "llama3-8b-shape Q4_0, batch 1, 512-token prompt, greedy decode (BASELINE config 3)", 512, 768
    if config == "70b":
        return (LLAMA3_70B, "llama3-70b-shape Q4_0, batch 1, 1024-token prompt, greedy decode (BASELINE config 5)",
                1024, 1280)
    if config == "tiny":
        sh = LlamaShape(**{**TINY.__dict__, "max_prompt": 512})
        return sh, "tiny Llama Q8_0 (BASELINE config 1 shape), batch 1", 512, 768
    raise ValueError(config)


def model_path(sh, config: str, rank: int, world: int, encoder=None) -> Path:
    """The synthetic GGUF of this config (written once per box, then reused). `encoder` encodes the
    quantized matrices: the product library's by default, the oracle's on the reference arm, which
    must not load the product; both are bit-exact with gguf-py, so the file is the same either way."""
    from ggml_compiler_b200.llm import build_llama_gguf

    CACHE.mkdir(parents=True, exist_ok=True)
    p = CACHE / f"{config}_{sh.weight_type}_seed0.gguf"
    if rank == 0 and not p.exists():
        tmp = p.with_suffix(f".part{os.getpid()}")
        t = time.time()
        build_llama_gguf(tmp, sh, seed=0, encoder=encoder)
        tmp.rename(p)
        print(f"[bench] wrote {p} ({p.stat().st_size / 1e9:.2f} GB) in {time.time() - t:.1f}s", file=sys.stderr)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    return p


def weight_bytes(sh) -> float:
    """Quantized weight bytes streamed per decode token (every projection + the output head)."""
    from ggml_compiler_b200.llm import llama_weights

    per = {"q4_0": 18 / 32, "q8_0": 34 / 32, "f16": 2, "f32": 4}
    tot = 0.0
    for _, hf, shape, typ in llama_weights(sh):
        if "embed_tokens" in hf:
            continue  # one row gathered per token
        tot += float(np.prod(shape)) * per[typ]
    return tot


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.out = device, None, None

    def __enter__(self):
        try:
            self.out = open(CACHE / f"clocks_{self.device}.csv", "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.out:
            self.out.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(", ") for r in (CACHE / f"clocks_{self.device}.csv").read_text().strip().splitlines()]
        except OSError:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = [r for r in rows if len(r) >= 9 and r[1].strip().isdigit()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_baseline(gguf: Path, sh, n_tokens: int, prompt: int, n_kv: int) -> dict:
    """The reference's CPU arithmetic for the path (oracle/, the C restatement of ggml's CPU code) on
    the host's cores, on the GPU arm's workload: greedy decode steps at positions prompt, prompt+1,
    ... with attention over n_kv cache rows. Prefilling `prompt` tokens on the CPU would take
    minutes, so the cache rows of the prompt positions are filled with seeded f16 values instead:
    a decode step's work does not depend on what the cache holds. One untimed step, then
    `n_tokens` timed."""
    import oracle
    from oracle.interp import OracleGenerator, Program

    p = Program(gguf)
    g = OracleGenerator(p)
    g.reset()
    rng = np.random.default_rng(1)
    for name in p.prog.get("state", []):
        cache = p.values[name].reshape(sh.kv_heads, -1, sh.hd)  # [Hkv, max_context, D] f16
        cache[:, :prompt] = (rng.standard_normal((sh.kv_heads, prompt, sh.hd), np.float32) * 0.5).astype(np.float16)
    g.n_past = prompt
    tok = int(rng.integers(0, sh.vocab))
    tok = int(np.argmax(g.feed([tok])))
    t = time.perf_counter()
    for _ in range(n_tokens):
        tok = int(np.argmax(g.feed([tok])))
    dt = time.perf_counter() - t
    return {"value": n_tokens / dt, "unit": "tok/s", "cores": oracle.lib().orc_get_threads(), "kind": "port",
            "sample": f"{n_tokens} greedy decode steps of the same model at positions {prompt + 1}.. (n_kv {n_kv}, "
                      f"the cache rows of a {prompt}-token prompt filled with seeded values), oracle/ C restatement "
                      f"of ggml's CPU arithmetic, {dt:.1f}s"}


SWEEP_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]  # weight [N x K]
SWEEP_M = [1, 8, 64, 512, 2048]


def sweep(args) -> None:
    """isolated quantized mul_mat (one-node programs through the C ABI), weights
    from N(0, 0.02) seed 0 as Q4_0 / Q8_0, activations N(0, 1). Each case prints one JSON line with
    the kernel's device time (profiled launch, L2 flushed by a 256 MB write before each rep) and its
    bytes / FLOPs rates. `--shape NxK --m M --wtype T` runs one case (the ncu captures use that)."""
    import torch

    from ggml_compiler_b200.gguf_write import BLOCKS
    from ggml_compiler_b200.programs import random_block_rows, write_mul_mat
    from ggml_compiler_b200.runtime import Model

    peak, peak_kind = peaks()
    tflops = None
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        tflops = float(json.loads(pk.read_text())["bf16_tflops"])
    shapes = [tuple(int(v) for v in args.shape.lower().split("x"))] if args.shape else SWEEP_SHAPES
    ms_ = [args.m] if args.m else SWEEP_M
    wts = [args.wtype] if args.wtype else ["q4_0", "q8_0"]
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    CACHE.mkdir(parents=True, exist_ok=True)
    for wt in wts:
        for N, Kd in shapes:
            rng = np.random.default_rng(0)
            w = None
            for M in ms_:
                p = CACHE / f"mm_{wt}_{N}x{Kd}_m{M}.gguf"
                if not p.exists():
                    if w is None and wt in ("iq4_nl", "q4_k", "q5_k", "q6_k"):  # no encoder: synthetic blocks
                        w = random_block_rows(wt, N, Kd, seed=0)
                    elif w is None:
                        w = rng.standard_normal((N, Kd), dtype=np.float32) * np.float32(0.02)
                    write_mul_mat(p, w, wt, M)
                x = np.random.default_rng(1).standard_normal((1, M, Kd), dtype=np.float32)
                with Model(p) as s:
                    run = s.entries["main"]
                    for _ in range(max(3, args.warmup)):
                        run(x=x)
                    s.profile(True)
                    for _ in range(args.steps):
                        flush.fill_(1.0)
                        torch.cuda.synchronize()
                        run(x=x)
                    ks = s.kernel_table()
                    s.profile(False)
                kinds = [k for k in ks if k.startswith(("gemv", "mul_mat"))]
                ms = sum(ks[k]["ms"] for k in kinds) / max(1, sum(ks[k]["launches"] for k in kinds))
                wbytes = N * Kd * BLOCKS[wt][1] / BLOCKS[wt][0]  # the format's stored bytes
                byts = wbytes + 4.0 * M * Kd + 4.0 * M * N
                flops = 2.0 * M * N * Kd
                print(json.dumps({"metric": "isolated quantized mul_mat (BASELINE config 2)", "kernel": "+".join(kinds),
                                  "wtype": wt, "N": N, "K": Kd, "M": M, "us": ms * 1000.0,
                                  "GB_s": byts / (ms / 1000.0) / 1e9, "hbm_frac": byts / (ms / 1000.0) / 1e9 / peak,
                                  "TFLOP_s": flops / (ms / 1000.0) / 1e12,
                                  "tensor_frac": (flops / (ms / 1000.0) / 1e12 / tflops) if tflops else None,
                                  "peak_source": f"{peak_kind} MEASURED_PEAKS.json", "reps": args.steps,
                                  "l2": "flushed before each rep (256 MB write)"}), flush=True)


ATTN_CASES = [(2048, 2048, "prefill"), (1, 768, "decode")]  # (query rows, n_kv): 8B shape, 32 / 8 heads, D 128


def attn(args) -> None:
    """Isolated flash_attn at the 8B shape (one-node programs through the C ABI): a 2048-row causal
    prefill over 2048 keys and one decode row over 768 keys (the 8B decode bench's n_kv, keys past
    position 520 hidden). The reference programs' mask value -65504 hides keys. One JSON line per
    case: the kernel's device time (profiled launch, L2 flushed before each rep), the FLOPs of the
    visible keys and the K/V bytes."""
    import torch

    from ggml_compiler_b200.gguf_write import write_gguf
    from ggml_compiler_b200.programs import single_node_program
    from ggml_compiler_b200.runtime import Model

    D, H, HKV = 128, 32, 8
    if args.prefill_attn == "tc":  # read when a model loads
        os.environ["GGML_COMPILER_B200_PREFILL_ATTN"] = "tc"
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    CACHE.mkdir(parents=True, exist_ok=True)
    for nq, nkv, kind in ATTN_CASES:
        rng = np.random.default_rng(3)
        q = rng.standard_normal((1, H, nq, D), dtype=np.float32)
        k = rng.standard_normal((1, HKV, nkv, D), dtype=np.float32).astype(np.float16)
        v = rng.standard_normal((1, HKV, nkv, D), dtype=np.float32).astype(np.float16)
        pos0 = nkv - nq if kind == "prefill" else 520
        m = np.zeros((nq, nkv), np.float32)
        for i in range(nq):
            m[i, pos0 + i + 1:] = -65504.0
        ins = [("q", "f32", [D, nq, H, 1], [1, H, nq, D]), ("k", "f16", [D, nkv, HKV, 1], [1, HKV, nkv, D]),
               ("v", "f16", [D, nkv, HKV, 1], [1, HKV, nkv, D]), ("mask", "f16", [nkv, nq, 1, 1], [1, 1, nq, nkv])]
        prog = single_node_program("flash_attn", ins, ["q", "k", "v", "mask"], "f32", [D, H, nq, 1], [1, nq, H, D],
                                   {"scale": float(1.0 / np.sqrt(D))})
        p = CACHE / f"attn_{kind}_{nq}x{nkv}.gguf"
        write_gguf(p, prog, [])
        feed = {"q": q, "k": k, "v": v, "mask": m.astype(np.float16)[None, None]}
        with Model(p) as s:
            run = s.entries["main"]
            for _ in range(max(3, args.warmup)):
                run(**feed)
            s.profile(True)
            for _ in range(args.steps):
                flush.fill_(1.0)
                torch.cuda.synchronize()
                run(**feed)
            ks = s.kernel_table()
            s.profile(False)
        fa = ks.get("flash_attn", {"ms": 0.0, "launches": 1})
        us = 1000.0 * fa["ms"] / max(1, fa["launches"])
        visible = sum(min(nkv, pos0 + i + 1) for i in range(nq))
        flops = 4.0 * H * D * visible
        kv_bytes = 2.0 * HKV * nkv * D * 2
        print(json.dumps({"metric": "isolated flash_attn (8B shape)", "case": kind, "rows": nq, "n_kv": nkv, "us": us,
                          "TFLOP_s_visible": flops / (us * 1e-6) / 1e12, "kv_GB_s": kv_bytes / (us * 1e-6) / 1e9,
                          "reps": args.steps, "l2": "flushed before each rep (256 MB write)",
                          "prefill_attn": args.prefill_attn if kind == "prefill" else None}), flush=True)


def batch_layers(args) -> None:
    """Batched decode at the 8B layer shape on a 2-layer model (d_model 4096, 32 / 8 heads, FFN 14336,
    vocab 2000, Q4_0 or --wtype): 8 sequences of 512 ids prefilled into KV-cache slots, then
    generate_batch steps. Small enough on the device (about 0.3 GB of weights) for full ncu
    captures of the batched kernels. One JSON line: batched decode tok/s and the step's weight rate."""
    from ggml_compiler_b200.llm import Decoder, LlamaShape, build_llama_gguf
    from ggml_compiler_b200.runtime import Model

    wt = args.wtype or "q4_0"
    sh = LlamaShape(layers=2, d_model=4096, heads=32, kv_heads=8, ffn=14336, vocab=2000, rope_theta=500000.0,
                    max_context=1024, max_prompt=512, weight_type=wt)
    CACHE.mkdir(parents=True, exist_ok=True)
    gguf = CACHE / f"layers2_8b_width_{wt}_seed3.gguf"
    if not gguf.exists():
        tmp = gguf.with_suffix(f".part{os.getpid()}")
        build_llama_gguf(tmp, sh, seed=3)
        tmp.rename(gguf)
    n, P = 8, 512
    with Model(gguf) as m:
        first, start = Decoder(m).fill_slots(np.random.default_rng(4).integers(0, sh.vocab, (n, P)).tolist())
        for _ in range(max(3, args.warmup)):
            m.generate_batch(first, start, 4)
        m.generate_batch(first, start, args.steps)
        ms = m.device_ms
    print(json.dumps({"metric": "batched decode at the 8B layer shape (2 layers)", "value": n * args.steps / (ms / 1000.0),
                      "unit": "tok/s", "batch": n, "steps": args.steps, "ms_per_step": ms / args.steps,
                      "weight_gb_s": weight_bytes(sh) / (ms / args.steps / 1000.0) / 1e9, "weights": wt}), flush=True)


def layers_decode(args) -> None:
    """Single-sequence decode at the 8B layer shape on a 2-layer model (d_model 4096, 32 / 8 heads,
    FFN 14336, vocab 2000) in any weight format (--wtype; the formats this library cannot encode
    get seeded synthetic blocks): 512 prompt ids, then greedy steps through the generate entry's
    device loop. One JSON line: tok/s, ms per step and per layer, the step's weight rate. Q4_0 /
    Q8_0 / q5_0 / iq4_nl groups run fused; q4_1 / q5_1 / K-quant groups run as separate ops."""
    from ggml_compiler_b200.llm import Decoder, LlamaShape, build_llama_gguf
    from ggml_compiler_b200.programs import random_block_rows
    from ggml_compiler_b200.runtime import Model, encode
    from ggml_compiler_b200.gguf_write import BLOCKS

    wt = args.wtype or "q4_0"
    sh = LlamaShape(layers=2, d_model=4096, heads=32, kv_heads=8, ffn=14336, vocab=2000, rope_theta=500000.0,
                    max_context=1024, max_prompt=512, weight_type=wt)

    def encoder(w, typ):
        if typ in ("iq4_nl", "q4_k", "q5_k", "q6_k"):
            return random_block_rows(typ, w.shape[0], w.shape[1], seed=w.shape[0] * 7 + w.shape[1])
        return encode(w, typ)

    CACHE.mkdir(parents=True, exist_ok=True)
    gguf = CACHE / f"layers2_8b_width_{wt}_seed3.gguf"
    if not gguf.exists():
        tmp = gguf.with_suffix(f".part{os.getpid()}")
        build_llama_gguf(tmp, sh, seed=3, encoder=encoder)
        tmp.rename(gguf)
    P, n = 512, max(8, args.steps)
    wbytes = 0.0
    from ggml_compiler_b200.llm import llama_weights
    for _, hf, shape, typ in llama_weights(sh):
        if "embed_tokens" not in hf:
            blk, size = BLOCKS[typ]
            wbytes += float(np.prod(shape)) * size / blk
    with Model(gguf) as m:
        d = Decoder(m)
        gen = m.entries["generate"]
        prompt = np.random.default_rng(1).integers(0, sh.vocab, P).tolist()
        ms = 0.0
        for rep in range(max(3, args.warmup) + 1):
            d.restart()
            first = int(np.argmax(d.prompt(prompt)))
            m.bind(max_new=n)
            gen.upload({"first": np.array([[first]], np.int32), "start": np.array([P], np.int32)})
            gen.launch()
            ms = m.device_ms
    step = ms / n
    print(json.dumps({"metric": "single-sequence decode at the 8B layer shape (2 layers)", "weights": wt,
                      "value": 1000.0 / step, "unit": "tok/s", "steps": n, "ms_per_step": step,
                      "us_per_layer_incl_head": 1000.0 * step / sh.layers, "weight_gb_s": wbytes / (step / 1000.0) / 1e9,
                      "weight_bytes_per_step": wbytes}), flush=True)


PREFILL_METRIC = "8B-shape Q8_0 prefill tok/s (8 sequences x 2048-token prompts); tensor-core TFLOP/s"


def prefill_bench(args) -> None:
    """BASELINE config 4's prefill: the 8B shape with Q8_0 projections, 8 random 2048-token prompts
    (seed 2), each prefilled in one 2048-row call (tensor-core GEMMs, flash prefill), then 64 greedy
    decode steps per sequence. The reference program is batch 1, so the 8 sequences run one after
    another. One JSON line: prefill tok/s (device time), e2e (host arrays through the prefill entry:
    tokens, positions and the f32 mask up, logits down), and the GEMMs' FLOP rate from a profiled
    pass against the measured dense bf16 peak (the int8 MMAs' nominal peak is twice that)."""
    import dataclasses

    import torch

    from ggml_compiler_b200.llm import LLAMA3_8B, Decoder, build_llama_gguf
    from ggml_compiler_b200.runtime import Model

    sh = dataclasses.replace(LLAMA3_8B, weight_type="q8_0", max_context=2304, max_prompt=2048)
    CACHE.mkdir(parents=True, exist_ok=True)
    gguf = CACHE / "8b_q8_0_ctx2304_seed0.gguf"
    if not gguf.exists():
        tmp = gguf.with_suffix(".part")
        build_llama_gguf(tmp, sh, seed=0)
        tmp.rename(gguf)
    n_seq, plen, n_dec = 8, 2048, 64
    prompts = np.random.default_rng(2).integers(0, sh.vocab, (n_seq, plen))
    if args.prefill_attn == "tc":  # read when the model loads
        os.environ["GGML_COMPILER_B200_PREFILL_ATTN"] = "tc"
    s = Model(gguf)
    g = Decoder(s)
    # warm-up: one sequence (plans and graphs for the 2048-row call and decode at n_kv 2304)
    g.restart()
    tok = int(np.argmax(g.prompt(prompts[0].tolist())))
    for _ in range(max(3, args.warmup)):
        tok = int(np.argmax(g.step(tok)))
    pre_dev = pre_wall = dec_dev = 0.0
    s.seq_slots(n_seq)
    first, single = [], []
    with Clocks(0) as clk:
        for i in range(n_seq):
            g.restart()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            tok = int(np.argmax(g.prompt(prompts[i].tolist())))
            pre_wall += time.perf_counter() - t0
            pre_dev += s.device_ms
            first.append(tok)
            s.seq_copy(i, -1)  # the sequence's prefilled state into its slot for the batched decode
            toks = []
            for _ in range(n_dec):
                tok = int(np.argmax(g.step(tok)))
                toks.append(tok)
                dec_dev += s.device_ms
            single.append(toks)
        # batched decode (include/ggml_compiler_b200.h): the 8 sequences in one step, greedy on the
        # device; a warm-up call first (plans and graphs; it writes the same cache rows again)
        start = np.full(n_seq, plen, np.int32)
        s.generate_batch(first, start, 3)
        got = s.generate_batch(first, start, n_dec)
        bat_dev = s.device_ms
    s.profile(True)  # the batched step's launches one by one, timed
    s.generate_batch(first, start, 4)
    kb = s.kernel_table()
    s.profile(False)
    # profiled pass over one prefill: the GEMM kernels' share and FLOP rate
    g.restart()
    s.profile(True)
    g.prompt(prompts[0].tolist())
    ks = s.kernel_table()
    s.profile(False)
    s.close()
    d, H, Hkv, D, F = sh.d_model, sh.heads, sh.kv_heads, sh.hd, sh.ffn
    gemm_flops = 2.0 * plen * d * (H * D + 2 * Hkv * D + d + 3 * F) * sh.layers + 2.0 * d * sh.vocab  # head: last row
    attn_flops = 4.0 * H * D * (plen * (plen + 1) / 2) * sh.layers  # QK^T and PV over the causal half
    mm = ks.get("mul_mat", {"ms": 0.0, "launches": 0})
    # algorithmic bytes of the call's GEMMs: Q8_0 weights (34 B per 32) and Q8_0 activation codes
    gemm_alg_bytes = (sh.layers * d * (H * D + 2 * Hkv * D + d + 3 * F) * (34 / 32)
                      + sh.layers * plen * (5 * d + H * D + F) * (34 / 32))
    total_ms = sum(v["ms"] for v in ks.values())
    pk = REPO / "MEASURED_PEAKS.json"
    tflops_peak = float(json.loads(pk.read_text())["bf16_tflops"]) if pk.exists() else 1590.0
    achieved = gemm_flops / (mm["ms"] / 1000.0) / 1e12 if mm["ms"] else 0.0
    value = n_seq * plen / (pre_dev / 1000.0)
    print(json.dumps({
        "metric": PREFILL_METRIC, "value": value, "unit": "tok/s", "n_gpus": 1, "steps": n_seq, "warmup": max(3, args.warmup),
        "ms_per_step": pre_dev / n_seq, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0 weights, int8 x int8 tcgen05.mma (kind::i8) block products, f32 scaling", "data": "synthetic",
        "config": {"workload": "llama3-8b-shape Q8_0, 8 x 2048-token prefill (one call each) + 64 decode steps each "
                               "(BASELINE config 4; batch 1 per call: the reference program has no batch dim)",
                   "layers": sh.layers, "d_model": d, "heads": H, "kv_heads": Hkv, "ffn": F, "vocab": sh.vocab,
                   "weights": "q8_0", "l2": "no flush: each call streams 7.5 GB of weights and GBs of activations",
                   "prefill_attn": ("tensor cores (mma.sync f16, within tolerance of the checker)" if args.prefill_attn == "tc"
                                    else "CUDA cores, bit-exact with the checker")},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tflops_peak, "unit": "TFLOP/s",
                     "frac": achieved / tflops_peak, "kernel": "mul_mat (gemm_tc)",
                     "traffic": GEMM_TRAFFIC_RATIO * gemm_alg_bytes / max(1, mm["launches"]),
                     "traffic_source": "DRAM bytes per launch = 1.0025 x algorithmic (weights + activation codes), the "
                                       "ratio of an ncu capture of the 4096x4096 M=512 Q4_0 GEMM, scaled to this "
                                       "call's GEMMs",
                     "peak_source": "measured bf16_tflops (MEASURED_PEAKS.json); int8 nominal peak is 2x",
                     "gemm_flops_per_call": gemm_flops, "attn_flops_per_call": attn_flops,
                     "gemm_share_of_call": mm["ms"] / total_ms if total_ms else None,
                     "call_tflops": (gemm_flops + attn_flops) / (pre_dev / n_seq / 1000.0) / 1e12,
                     "call_frac": (gemm_flops + attn_flops) / (pre_dev / n_seq / 1000.0) / 1e12 / tflops_peak},
        "e2e": {"value": n_seq * plen / pre_wall, "unit": "tok/s", "h2d_bytes_per_step": plen * 8 + plen * plen * 4,
                "d2h_bytes_per_step": 4 * sh.vocab},
        "decode_tok_s": n_seq * n_dec / (dec_dev / 1000.0),
        "batched_decode": {
            "value": n_seq * n_dec / (bat_dev / 1000.0), "unit": "tok/s", "batch": n_seq, "steps": n_dec,
            "ms_per_step": bat_dev / n_dec,
            "weight_gb_s": weight_bytes(sh) / (bat_dev / n_dec / 1000.0) / 1e9,
            "vs_batch1": (n_seq * n_dec / (bat_dev / 1000.0)) / (n_seq * n_dec / (dec_dev / 1000.0)),
            "tokens_equal_batch1": bool(np.array_equal(np.asarray(got).T, np.asarray(single))),
            "kernel_breakdown_ms_per_step": {k: v["ms"] / 4 for k, v in sorted(kb.items(), key=lambda kv: -kv[1]["ms"])},
            "how": "generate_batch: one step decodes all 8 sequences (8-row GEMVs, attention over 8 KV slots), "
                   "greedy tokens fed back on the device; device time of the 64 steps"},
        "gpu_launches": int(sum(v["launches"] for v in ks.values()) * n_seq),
        "clocks": clk.summary(),
        "kernel_breakdown_ms_per_call": {k: v["ms"] for k, v in sorted(ks.items(), key=lambda kv: -kv[1]["ms"])},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="8b", choices=["8b", "70b", "tiny", "sweep", "prefill", "attn", "batch", "layers"])
    ap.add_argument("--no-tp-probe", action="store_true",
                    help="N>1 replicas: skip the extra tensor-parallel measurement of the same model")
    ap.add_argument("--prefill-attn", default="exact", choices=["exact", "tc"],
                    help="prefill: attention on the CUDA cores bit-exact with the checker (exact) or on the tensor cores (tc)")
    ap.add_argument("--shape", default=None, help="sweep: one weight shape NxK")
    ap.add_argument("--m", type=int, default=None, help="sweep: one activation row count")
    ap.add_argument("--wtype", default=None,
                    choices=["q4_0", "q8_0", "q4_1", "q5_0", "q5_1", "iq4_nl", "q4_k", "q5_k", "q6_k"],
                    help="sweep: one weight type (the other block formats run only when named)")
    ap.add_argument("--parallel", default="replicas", choices=["tp", "replicas"],
                    help="N>1: N independent sequences (replicas), or one sequence tensor-parallel over the N GPUs (tp)")
    ap.add_argument("--cpu-tokens", type=int, default=12)  # about 10 s of the oracle on 16 host threads
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="decode only: prefill and warm up, then run this many device-loop decode steps between "
                         "cudaProfilerStart/Stop (for `ncu --profile-from-start off`) and exit without a JSON line")
    args = ap.parse_args()

    if args.config == "sweep":
        if args.steps == ap.get_default("steps"):
            args.steps = 10
        sweep(args)
        return
    if args.config == "prefill":
        prefill_bench(args)
        return
    if args.config == "attn":
        if args.steps == ap.get_default("steps"):
            args.steps = 10
        attn(args)
        return
    if args.config == "layers":
        if args.steps == ap.get_default("steps"):
            args.steps = 64
        layers_decode(args)
        return
    if args.config == "batch":
        if args.steps == ap.get_default("steps"):
            args.steps = 16
        batch_layers(args)
        return
    decode_bench(args)


def decode_bench(args) -> None:
    """BASELINE config 3 (or the 70B shape): greedy decode tok/s, see the module docstring."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    sh, workload, P, NKV = shape_for(args.config)
    K, W = min(args.steps, NKV - P), max(3, args.warmup)
    metric = {"70b": "70B-shape Q4_0 decode tok/s; quant-GEMV HBM GB/s as % of B200 peak",
              "tiny": "tiny-Llama (BASELINE config 1 shape) Q8_0 decode tok/s"}.get(args.config, METRIC)
    wgb = weight_bytes(sh) / 1e9
    tp = world > 1 and args.parallel == "tp"
    config = {"workload": workload, "layers": sh.layers, "d_model": sh.d_model, "heads": sh.heads,
              "kv_heads": sh.kv_heads, "ffn": sh.ffn, "vocab": sh.vocab, "weights": sh.weight_type, "batch": 1,
              "prompt": P, "decode_tokens": K, "n_kv": NKV,
              "l2": f"no flush: the decode step streams all weights ({wgb:.1f} GB) through a 126 MB L2",
              "parallelism": (f"tp{world}: rows / heads split, exchanges over NVLink peer memory" if tp
                              else f"replicas x{world}" if world > 1 else "single GPU")}
    dtype = f"{sh.weight_type} weights, int8 x int{4 if sh.weight_type == 'q4_0' else 8} block dots, f32 sums"

    if args.impl == "reference":
        # the reference's CPU arithmetic (oracle port) on the host cores; rank 0 only, no product code
        if rank != 0:
            return
        import oracle

        gguf = model_path(sh, args.config, 0, 1, encoder=oracle.quantize)
        n = max(1, min(K, args.cpu_tokens))
        cb = cpu_baseline(gguf, sh, n, P, NKV)
        print(json.dumps({"impl": "reference", "metric": metric, "value": cb["value"], "unit": "tok/s",
                          "n_gpus": args.gpus, "steps": n, "warmup": 1, "ms_per_step": 1000.0 / cb["value"],
                          "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
                          "dtype": dtype, "data": "synthetic", "config": config, "cpu_baseline": cb,
                          "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return

    import ctypes

    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    torch.cuda.set_device(local)
    from ggml_compiler_b200.llm import Decoder
    from ggml_compiler_b200.runtime import BackendError, Model, load_library, torch_all_gather

    lib = load_library()
    gguf = model_path(sh, args.config, rank, world)
    m = Model(gguf, device=local)
    if tp:
        m.join_tensor_parallel(rank, world, torch_all_gather())
    seqs = 1 if tp else world  # sequences decoded by the whole job
    stream = torch.cuda.ExternalStream(m.stream, device=torch.device("cuda", local))
    d = Decoder(m)
    prompt = np.random.default_rng(1).integers(0, sh.vocab, P).tolist()
    gen = m.entries["generate"]

    def prefill() -> int:
        d.restart()
        return int(np.argmax(d.prompt(prompt)))

    def generate(first: int, n: int) -> float:
        m.bind(max_new=n)
        gen.upload({"first": np.array([[first]], np.int32), "start": np.array([P], np.int32)})
        gen.launch()
        return m.device_ms

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], device="cuda")
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # warm-up: prefill + W device-loop steps (plans and graphs for the decode n_kv)
    first = prefill()
    generate(first, W)
    if args.profile_steps:
        first = prefill()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        generate(first, args.profile_steps)
        torch.cuda.profiler.stop()
        m.close()
        return

    # timed: K decode steps in the device loop, inputs resident
    barrier()
    with Clocks(local) as clk:
        dev_ms = generate(first, K)
    barrier()
    dev_ms = max_over_ranks(dev_ms)
    value = seqs * K / (dev_ms / 1000.0)

    # e2e: one `decode` entry per token through the C ABI, host buffers (pinned) both ways
    tok_h = torch.empty((1, 1), dtype=torch.int32, pin_memory=True).numpy()
    pos_h = torch.empty(1, dtype=torch.int32, pin_memory=True).numpy()
    mask_h = torch.empty((1, 1, 1, NKV), dtype=torch.float32, pin_memory=True).numpy()
    out_h = torch.empty((1, 1, sh.vocab), dtype=torch.float32, pin_memory=True).numpy()
    mask_dims = (ctypes.c_int64 * 4)(*mask_h.shape)
    cols = np.arange(NKV)

    def check(rc: int) -> None:
        if rc != 0:
            raise BackendError(lib.ggml_compiler_last_error().decode())

    def e2e_step(tok: int, p: int) -> int:
        tok_h[0, 0] = tok
        pos_h[0] = p
        mask_h[0, 0, 0] = np.where(cols <= p, np.float32(0.0), np.float32(-np.inf))
        check(lib.ggml_compiler_set_input_shape(m.handle, b"mask1", 4, mask_dims))
        for name, arr in ((b"token", tok_h), (b"position", pos_h), (b"mask1", mask_h)):
            check(lib.ggml_compiler_set_input(m.handle, name, arr.ctypes.data, arr.nbytes))
        check(lib.ggml_compiler_run_entry(m.handle, b"decode"))
        check(lib.ggml_compiler_get_output(m.handle, b"logits1", out_h.ctypes.data, out_h.nbytes))
        return int(np.argmax(out_h))

    tok = prefill()
    for i in range(W):
        tok = e2e_step(tok, P + i)
    tok = prefill()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    w0 = time.perf_counter()
    for i in range(K):
        tok = e2e_step(tok, P + i)
    ev1.record(stream)
    ev1.synchronize()
    wall = time.perf_counter() - w0
    e2e_value = seqs * K / (max_over_ranks(max(ev0.elapsed_time(ev1), wall * 1000.0)) / 1000.0)

    # roofline: a profiled pass over the same decode steps (each launch timed with CUDA events on
    # the model's stream, no graphs), per kernel family
    first = prefill()
    m.profile(True)
    n_prof = min(K, 16)
    generate(first, n_prof)
    ks = m.kernel_table()
    m.profile(False)
    gemv_kinds = [k for k in ks if k.startswith(("gemv", "decode_")) or k == "mul_mat"]
    gemv_ms = sum(ks[k]["ms"] for k in gemv_kinds)
    gemv_bytes = sum(ks[k]["bytes"] for k in gemv_kinds)
    gemv_launches = sum(ks[k]["launches"] for k in gemv_kinds)
    total_ms = sum(v["ms"] for v in ks.values())
    launches_per_step = sum(v["launches"] for v in ks.values()) / n_prof
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms / 1000.0) / 1e9 if gemv_ms else 0.0
    step_bytes = weight_bytes(sh) / (world if tp else 1)

    out = {
        "metric": metric, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": dev_ms / K, "higher_is_better": True, "scaling": "strong" if tp else "weak",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if peak else None,
                     "traffic": GEMV_TRAFFIC_RATIO * gemv_bytes / max(1, gemv_launches),
                     "traffic_source": "DRAM bytes per launch = 1.0048 x algorithmic, the ratio of an ncu capture "
                                       "of the 4096x4096 Q4_0 GEMV, scaled to this mix of launches",
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "kernel": "+".join(gemv_kinds),
                     "bytes_per_launch": gemv_bytes / max(1, gemv_launches),
                     "mean_launch_us": 1000.0 * gemv_ms / max(1, gemv_launches),
                     "share_of_step": gemv_ms / total_ms if total_ms else None,
                     "step_weight_bytes": step_bytes,
                     "step_achieved_gbs": step_bytes / (dev_ms / K / 1000.0) / 1e9,
                     "step_hbm_frac": step_bytes / (dev_ms / K / 1000.0) / 1e9 / peak,
                     "frac_of_spec_8000_gbs": achieved / 8000.0},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4 + 4 + 4 * NKV,
                "d2h_bytes_per_step": 4 * sh.vocab, "wall_ms": wall * 1000.0},
        "gpu_launches": int(round(launches_per_step * K + 2 * K)),
        "clocks": clk.summary(),
        "kernel_breakdown_ms_per_step": {k: v["ms"] / n_prof for k, v in sorted(ks.items(), key=lambda kv: -kv[1]["ms"])},
    }
    if not tp and world == 1:
        # batched decode (include/ggml_compiler_b200.h): 8 sequences of the same model and prompt
        # length, one step for all of them, greedy tokens fed back on the device
        nbat, bsteps = 8, min(64, NKV - P)
        bprompts = [np.random.default_rng(10 + i).integers(0, sh.vocab, P).tolist() for i in range(nbat)]
        bfirst, bstart = d.fill_slots(bprompts)
        m.generate_batch(bfirst, bstart, 3)  # plans and graphs
        m.generate_batch(bfirst, bstart, bsteps)
        bms = m.device_ms
        out["batched_decode"] = {
            "value": nbat * bsteps / (bms / 1000.0), "unit": "tok/s", "batch": nbat, "steps": bsteps,
            "ms_per_step": bms / bsteps, "vs_batch1": (nbat * bsteps / (bms / 1000.0)) / value,
            "weight_gb_s": weight_bytes(sh) / (bms / bsteps / 1000.0) / 1e9,
            "how": "8 sequences prefilled (512 ids each) into KV-cache slots, then generate_batch: one step decodes "
                   "all 8 (tensor-core GEMVs over 8 rows, attention over the 8 slots), device time of the steps"}
    if world > 1 and not tp and not args.no_tp_probe:
        # the same model decoded as one sequence split over the N GPUs (the tensor-parallel path:
        # rows / heads per rank, exchanges over NVLink peer memory), beside the N replicas above
        try:
            m.join_tensor_parallel(rank, world, torch_all_gather())
            tfirst = prefill()
            generate(tfirst, W)
            tfirst = prefill()
            barrier()
            tms = generate(tfirst, K)
            barrier()
            tms = max_over_ranks(tms)
            out["tensor_parallel"] = {
                "value": K / (tms / 1000.0), "unit": "tok/s", "ranks": world, "steps": K, "ms_per_step": tms / K,
                "vs_one_replica": (K / (tms / 1000.0)) / (value / world),
                "how": "one sequence, rows and heads split over the ranks, four exchanges per layer over NVLink "
                       "peer memory (bit-exact with one GPU); the headline value is the N replicas"}
        except Exception as e:  # reported beside the headline number, which stands on its own
            out["tensor_parallel"] = {"value": None, "error": str(e)[:200]}
    m.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline(gguf, sh, max(1, min(K, args.cpu_tokens)), P, NKV)
        except Exception as e:  # the baseline is reported, not required for the GPU number
            out["cpu_baseline"] = {"value": None, "unit": "tok/s", "error": str(e)[:200]}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
