"""One rank of the tensor-parallel GPU test (test_gpu_tp.py), run as its own process:

    python tests/tp_worker.py MODEL.gguf OUT_DIR RANK WORLD PORT CASE.json
    python tests/tp_worker.py MODEL.gguf OUT_DIR RANK WORLD PORT absent-peer

Loads the model on GPU RANK, joins the group (handles moved by torch.distributed over gloo on
127.0.0.1), feeds the case's chunks and greedy-decodes, and saves every step's logits and the tokens
to OUT_DIR/rank{RANK}.npz.

absent-peer: every rank prefills (no exchange), then rank 0 alone runs a decode step while the
other ranks wait on the host, alive, with their windows mapped; rank 0's first exchange waits for
flags that nothing sets, gives up after GGML_COMPILER_B200_TP_TIMEOUT_MS and the run fails. Rank 0
writes the error (or "no error") to OUT_DIR/rank0.txt; then all ranks meet and exit."""

import json
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(REPO), str(REPO / "ggml-compiler_b200")]


def run_case(sess, case: dict) -> dict:
    """Logits after each chunk (last row), greedy tokens through the host loop and the device loop."""
    from ggml_compiler_b200.llm import Decoder

    g = Decoder(sess)
    g.restart()
    logits = []
    for c in case["chunks"]:
        logits.append(np.asarray(g.prompt(c), np.float32))
    toks = g.greedy(case["prompt"], case["max_new"])
    dev = g.greedy(case["prompt"], case["max_new"], on_device=True)
    return {"logits": np.stack(logits), "tokens": np.array(toks), "device_tokens": np.array(dev)}


def main() -> None:
    import torch.distributed as dist

    from ggml_compiler_b200.runtime import Model, torch_all_gather

    path, out, rank, world, port, case = sys.argv[1], Path(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), sys.argv[5], sys.argv[6]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        sess = Model(path, device=rank)
        sess.join_tensor_parallel(rank, world, torch_all_gather())
        if case == "absent-peer":
            from ggml_compiler_b200.llm import Decoder
            from ggml_compiler_b200.runtime import BackendError

            g = Decoder(sess)
            g.restart()
            g.prompt(list(range(1, 17)))  # 16 rows: the prefill path, which exchanges nothing
            if rank == 0:
                try:
                    g.step(5)
                    outcome = "no error"
                except BackendError as e:
                    outcome = str(e)
                (out / "rank0.txt").write_text(outcome)
        else:
            res = run_case(sess, json.loads(Path(case).read_text()))
            np.savez(out / f"rank{rank}.npz", **res)
        dist.barrier()  # no rank frees its window while a peer may still push into it
        sess.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
