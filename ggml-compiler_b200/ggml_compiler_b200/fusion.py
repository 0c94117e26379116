"""Emitter fusion marks: the program-side half of the fused decode kernels.

The reference compiler's emitter (ggml_compiler/emit/gguf_runtime.py:117-202, build_program_json)
writes one JSON node per ggml op. This pass runs over that program JSON (format 3) after it is
built and adds an optional `"fuse": "<kind>.<n>"` key to every node of a group the B200 backend
runs as one fused kernel; a runtime that does not know the key ignores it, so the program still
runs on the reference's own ggml CPU runtime unchanged. The groups, by the nodes they cover (the
layer the reference emits at -O2/-O3 with fuse_rms_norm, fuse_glu, fuse_rope and the f16 KV cache):

    qkv    rms_norm -> mul(weight) -> views -> 3 x mul_mat -> views -> rope(q), rope(k) -> views ->
           set_rows(K cache), views -> set_rows(V cache)         (the views from rope(q) to the
           attention stay outside: attention reads them after the group)
    glu    rms_norm -> mul(weight) -> views -> 2 x mul_mat -> views -> swiglu
    head   rms_norm -> mul(weight) -> views -> 1 x mul_mat
    resid  mul_mat -> views -> add(residual, .)

A group is marked only if every node in it, other than the values it defines for later nodes, is
read only inside the group and is not a stage output. When a stage carries marks the backend fuses
exactly the marked groups (csrc/gc_fuse.cpp checks each against the shapes and strides its kernels
take, and runs a group it cannot take as separate ops); a stage without marks is matched by the
backend itself."""

from __future__ import annotations

import copy
from typing import Any

VIEW_OPS = ("reshape", "view", "permute")


class _Stage:
    def __init__(self, stage: dict[str, Any]):
        self.nodes = stage["nodes"]
        self.idx = {n["id"]: i for i, n in enumerate(self.nodes)}
        self.readers: list[list[int]] = [[] for _ in self.nodes]
        for i, n in enumerate(self.nodes):
            for s in n["src"]:
                if s in self.idx:
                    self.readers[self.idx[s]].append(i)
        self.outputs = set(stage.get("outputs", []))
        self.taken: set[int] = set()

    def op(self, i: int) -> str:
        return self.nodes[i]["op"]

    def reach(self, i: int) -> tuple[list[int], list[int]]:
        """Non-view readers reached from node i through views, and the views passed on the way."""
        views: list[int] = []
        terms: list[int] = []

        def walk(j: int) -> None:
            for r in self.readers[j]:
                if self.op(r) in VIEW_OPS:
                    views.append(r)
                    walk(r)
                else:
                    terms.append(r)

        walk(i)
        return views, terms

    def chain(self, frm: int, vid: str) -> list[int] | None:
        """The view nodes from node `frm` to value `vid`, or None if `vid` is not a view chain of it."""
        out: list[int] = []
        cur = self.idx.get(vid, -1)
        while cur != frm:
            if cur < 0 or self.op(cur) not in VIEW_OPS:
                return None
            out.append(cur)
            cur = self.idx.get(self.nodes[cur]["src"][0], -1)
        return out[::-1]

    def closed(self, group: list[int], outs: set[int]) -> bool:
        inside = set(group)
        for x in group:
            if x in outs:
                continue
            if self.nodes[x]["id"] in self.outputs:
                return False
            if any(r not in inside for r in self.readers[x]):
                return False
        return True


def _is_weight(name: str, weight_types: dict[str, str] | None) -> bool:
    """A GGUF tensor (not a node id or stage parameter) that a fused GEMV streams: Q4_0 or Q8_0, or
    q5_0 / iq4_nl, which the backend expands into Q8_0 at load."""
    if name.startswith("%") or name.startswith("a."):
        return False
    return weight_types is None or weight_types.get(name) in ("q4_0", "q8_0", "q5_0", "iq4_nl")


def _norm_in(st: _Stage, i: int, wt: dict[str, str] | None) -> tuple[int, list[int], list[int]] | None:
    """rms_norm -> mul(weight) -> views -> mul_mats reading the normalised rows: (mul, views, mul_mats)."""
    n = st.nodes[i]
    if n["op"] != "rms_norm" or n["id"] in st.outputs or len(st.readers[i]) != 1:
        return None
    j = st.readers[i][0]
    mul = st.nodes[j]
    if mul["op"] != "mul" or mul["src"][0] != n["id"] or mul["id"] in st.outputs or mul["src"][1] in st.idx:
        return None
    views, terms = st.reach(j)
    if not terms or any(st.nodes[v]["id"] in st.outputs for v in views):
        return None
    for t in terms:
        mm = st.nodes[t]
        if mm["op"] != "mul_mat" or not _is_weight(mm["src"][0], wt) or st.chain(j, mm["src"][1]) is None:
            return None
    return j, views, terms


def _mark_stage(stage: dict[str, Any], wt: dict[str, str] | None) -> int:
    st = _Stage(stage)
    groups: list[tuple[str, list[int]]] = []

    def claim(kind: str, group: list[int]) -> None:
        g = sorted(set(group))
        if any(x in st.taken for x in g):
            return
        st.taken.update(g)
        groups.append((kind, g))

    for i in range(len(st.nodes)):
        if i in st.taken:
            continue
        m = _norm_in(st, i, wt)
        if m is None:
            continue
        j, in_views, mms = m
        base = [i, j] + in_views
        if len(mms) == 3:
            group = list(base)
            roles: dict[str, int] = {}
            ok = True
            for mmi in mms:
                views, terms = st.reach(mmi)
                if len(terms) != 1:
                    ok = False
                    break
                t = terms[0]
                if st.op(t) == "set_rows":
                    roles["v"], roles["sv"] = mmi, t
                elif st.op(t) == "rope":
                    v2, t2 = st.reach(t)
                    if len(t2) != 1:
                        ok = False
                        break
                    if st.op(t2[0]) == "set_rows":
                        roles["k"], roles["rk"], roles["sk"] = mmi, t, t2[0]
                        group += v2
                    elif st.op(t2[0]) == "flash_attn":
                        roles["q"], roles["rq"] = mmi, t
                    else:
                        ok = False
                        break
                else:
                    ok = False
                    break
                group += views + [mmi]
            if not ok or not all(r in roles for r in ("q", "k", "v")):
                continue
            group += [roles["rq"], roles["rk"], roles["sk"], roles["sv"]]
            if st.closed(group, {roles["rq"], roles["sk"], roles["sv"]}):
                claim("qkv", group)
        elif len(mms) == 2:
            group = list(base)
            sw = None
            ok = True
            for mmi in mms:
                views, terms = st.reach(mmi)
                if len(terms) != 1 or st.op(terms[0]) != "swiglu" or (sw is not None and terms[0] != sw):
                    ok = False
                    break
                sw = terms[0]
                group += views + [mmi]
            if not ok or sw is None:
                continue
            group.append(sw)
            if st.closed(group, {sw}):
                claim("glu", group)
        elif len(mms) == 1:
            group = base + [mms[0]]
            if st.closed(group, {mms[0]}):
                claim("head", group)

    for i, n in enumerate(st.nodes):
        if i in st.taken or n["op"] != "mul_mat" or not _is_weight(n["src"][0], wt):
            continue
        views, terms = st.reach(i)
        if len(terms) != 1 or st.op(terms[0]) != "add":
            continue
        add = st.nodes[terms[0]]
        if st.chain(i, add["src"][1]) is None or st.chain(i, add["src"][0]) is not None:
            continue
        group = [i, terms[0]] + views
        if not st.closed(group, {terms[0]}):
            continue
        if st.idx.get(add["src"][0], -1) >= i:  # the residual must exist when the group runs
            continue
        claim("resid", group)

    count: dict[str, int] = {}
    for kind, g in sorted(groups, key=lambda kg: kg[1][0]):
        k = count.get(kind, 0)
        count[kind] = k + 1
        for x in g:
            st.nodes[x]["fuse"] = f"{kind}.{k}"
    return len(groups)


def mark_fusion_groups(program: dict[str, Any], weight_types: dict[str, str] | None = None,
                       in_place: bool = False) -> dict[str, Any]:
    """The program with `"fuse"` marks on the nodes of every fusable group, stage by stage.
    `weight_types` (GGUF tensor name -> storage type) limits the matmul groups to Q4_0 / Q8_0
    weights; without it every GGUF tensor operand counts."""
    out = program if in_place else copy.deepcopy(program)
    for stage in out["stages"]:
        for n in stage["nodes"]:
            n.pop("fuse", None)
        _mark_stage(stage, weight_types)
    return out


def fusion_groups(program: dict[str, Any]) -> dict[str, dict[str, list[str]]]:
    """Per stage: mark -> the node ids that carry it."""
    res: dict[str, dict[str, list[str]]] = {}
    for stage in program["stages"]:
        marks: dict[str, list[str]] = {}
        for n in stage["nodes"]:
            if "fuse" in n:
                marks.setdefault(n["fuse"], []).append(n["id"])
        res[stage["name"]] = marks
    return res
