"""Emitter fusion marks (host side, no GPU): the pass over the reference compiler's program JSON
(ggml_compiler/emit/gguf_runtime.py:117-202 writes it) marks, per decoder layer, the four groups the
backend fuses (QKV + rope + KV-cache write, gate/up + SwiGLU, and the two matmul + residual adds)
and the output head; the marks are the only change to the program; the GGUF writer stores them."""

import collections
import json

import pytest
from conftest import GOLDEN

from ggml_compiler_b200.fusion import fusion_groups, mark_fusion_groups
from ggml_compiler_b200.llm import LlamaShape, build_llama_gguf, llama_program, llama_weights

GROUP_OPS = {  # non-view ops of each group kind
    "qkv": {"rms_norm": 1, "mul": 1, "mul_mat": 3, "rope": 2, "set_rows": 2},
    "glu": {"rms_norm": 1, "mul": 1, "mul_mat": 2, "swiglu": 1},
    "head": {"rms_norm": 1, "mul": 1, "mul_mat": 1},
    "resid": {"mul_mat": 1, "add": 1},
}


def strip(program):
    out = json.loads(json.dumps(program))
    for s in out["stages"]:
        for n in s["nodes"]:
            n.pop("fuse", None)
    return out


@pytest.mark.parametrize("fixture,layers", [("ref_program_gqa2.json", 2), ("ref_program_config1.json", 4)])
def test_marks_on_reference_programs(fixture, layers):
    ref = json.loads((GOLDEN / fixture).read_text())["program"]
    marked = mark_fusion_groups(ref)
    assert strip(marked) == ref  # nothing but the marks changes
    assert "fuse" not in json.dumps(ref)  # and the input is left alone
    for stage in marked["stages"]:
        nodes = {n["id"]: n for n in stage["nodes"]}
        groups = fusion_groups(marked)[stage["name"]]
        kinds = collections.Counter(m.split(".")[0] for m in groups)
        assert kinds == {"qkv": layers, "glu": layers, "resid": 2 * layers, "head": 1}, stage["name"]
        for mark, ids in groups.items():
            ops = collections.Counter(nodes[i]["op"] for i in ids if nodes[i]["op"] not in ("reshape", "view", "permute"))
            assert ops == GROUP_OPS[mark.split(".")[0]], (stage["name"], mark, ops)
            # a group's inner values are read only inside it; its outputs are the last op of each chain
            inside = set(ids)
            readers = collections.defaultdict(list)
            for n in stage["nodes"]:
                for s in n["src"]:
                    readers[s].append(n["id"])
            for i in ids:
                outside = [r for r in readers[i] if r not in inside]
                if outside:
                    assert nodes[i]["op"] in ("rope", "set_rows", "swiglu", "mul_mat", "add"), (mark, i, outside)
        unmarked = [n["op"] for n in stage["nodes"] if "fuse" not in n]
        assert unmarked.count("flash_attn") == layers and "mul_mat" not in unmarked


def test_marks_need_block_quantized_weights():
    ref = json.loads((GOLDEN / "ref_program_gqa2.json").read_text())["program"]
    f16 = {n: "f16" for s in ref["stages"] for x in s["nodes"] for n in x["src"] if n.startswith("w.")}
    assert all(not g for g in fusion_groups(mark_fusion_groups(ref, f16)).values())
    q8 = dict.fromkeys(f16, "q8_0")
    assert fusion_groups(mark_fusion_groups(ref, q8)) == fusion_groups(mark_fusion_groups(ref))


def test_gguf_writer_stores_marks(tmp_path):
    import gguf

    sh = LlamaShape(layers=2, d_model=256, heads=4, kv_heads=2, ffn=512, vocab=128, max_context=768, max_prompt=64)
    for marks in (True, False):
        path = tmp_path / f"m{int(marks)}.gguf"
        build_llama_gguf(path, sh, fusion_marks=marks)
        f = gguf.GGUFReader(str(path)).fields["ggml_compiler.program"]
        prog = json.loads(bytes(f.parts[f.data[0]]).decode())
        want = llama_program(sh)[0]
        if marks:
            assert prog == mark_fusion_groups(want, {g: t for g, _, _, t in llama_weights(sh)})
            assert strip(prog) == want
        else:
            assert prog == want


def test_no_mark_when_a_group_value_escapes():
    """A group whose inner value is read outside it (here: the normed rows also feed a stage output,
    and a gate/up product read by a later node) is not marked; the rest of the layer still is."""
    ref = json.loads((GOLDEN / "ref_program_gqa2.json").read_text())["program"]
    prog = json.loads(json.dumps(ref))
    st = next(s for s in prog["stages"] if s["name"] == "decode")
    nodes = st["nodes"]
    marked = fusion_groups(mark_fusion_groups(prog))["decode"]
    qkv0 = set(marked["qkv.0"])
    mul = next(n for n in nodes if n["id"] in qkv0 and n["op"] == "mul")
    st["outputs"] = st["outputs"] + [mul["id"]]  # the normed rows become a stage output
    glu0 = set(marked["glu.0"])
    gate = next(n for n in nodes if n["id"] in glu0 and n["op"] == "mul_mat")
    nodes.append({"id": f"%{len(nodes)}", "op": "cont", "src": [gate["id"]], "type": "f32", "ne": gate["ne"], "p": {}})
    again = fusion_groups(mark_fusion_groups(prog))["decode"]
    kinds = collections.Counter(m.split(".")[0] for m in again)
    assert kinds == {"qkv": 1, "glu": 1, "resid": 4, "head": 1}
    assert not (set().union(*again.values()) & (qkv0 | glu0))


def test_marking_is_idempotent_and_does_not_touch_input():
    ref = json.loads((GOLDEN / "ref_program_config1.json").read_text())["program"]
    once = mark_fusion_groups(ref)
    assert mark_fusion_groups(once) == once
    assert "fuse" not in json.dumps(ref)
