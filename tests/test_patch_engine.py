"""The engine patch recipe (rabbit2_b200/engine/patch_engine.py) on a synthetic
source: every edit lands at its anchor line, the replaced prompt-loop header is
replaced, and a missing or repeated anchor stops the recipe instead of patching the
wrong place.  (The real engine source is patched and built by
rabbit2_b200/engine/Makefile; test_engine.py runs the result.)"""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
spec = importlib.util.spec_from_file_location("patch_engine", os.path.join(ROOT, "rabbit2_b200", "engine", "patch_engine.py"))
patch_engine = importlib.util.module_from_spec(spec)
spec.loader.exec_module(patch_engine)


def synthetic_source():
    anchors = [a for a, _, _ in patch_engine.INSERTIONS]
    # every anchor once, in the order of the insertions, with filler lines between;
    # forward()'s prologue and attention half around their anchors
    lines = []
    for i, a in enumerate(dict.fromkeys(anchors)):
        if a == patch_engine.HOIST_END:
            lines += [patch_engine.HOIST_BEGIN, "        attention_body();"]
        lines += [f"/* filler {i} */", a]
        if a == patch_engine.FORWARD:
            lines += ["    const int prologue_local = 1;", patch_engine.HOIST_PROLOGUE_END]
    return "\n".join(lines) + "\n", anchors


def test_every_edit_lands_at_its_anchor():
    src, anchors = synthetic_source()
    out = patch_engine.patch(src)
    for anchor, where, text in patch_engine.INSERTIONS:
        if where == "replace":
            assert anchor + "\n" not in out
            assert text in out
        elif where == "before":
            assert text + anchor in out
        else:
            assert anchor + "\n" + text in out
    assert '#include "rbt_engine_hook.h"' in out
    assert "rbt_engine_prefill(&m, &s, tokens, nt, routing, fl, fr)" in out
    assert "for (int i = rbt_pre_ ? nt : 0; i < nt; i++) {" in out
    # the hoisted attention half: forward()'s prologue and attention lines, before the hook's include
    hoisted = out[out.index("static void rbt_engine_attention_block("):out.index('#include "rbt_engine_hook.h"')]
    assert "    const int prologue_local = 1;" in hoisted and "        attention_body();" in hoisted
    assert "/* ---- MoE feed-forward ---- */" not in hoisted


def test_missing_or_repeated_anchor_stops_the_recipe():
    src, anchors = synthetic_source()
    with pytest.raises(SystemExit, match="anchor found 0 times"):
        patch_engine.patch(src.replace(anchors[-1] + "\n", ""))
    with pytest.raises(SystemExit, match="anchor found 2 times"):
        patch_engine.patch(src + anchors[-1] + "\n")
