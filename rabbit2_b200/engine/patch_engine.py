"""Build recipe: the RABBIT2 engine with its MoE block (or its whole forward) on the GPU.

    python rabbit2_b200/engine/patch_engine.py <rabbit2.c> <out.c>

Writes a copy of the engine source (rabbit2/src/rabbit2.c) with these edits and
nothing else changed: the include of rbt_engine_hook.h, its CLI flags, its init
call, the whole-forward and MoE-block calls in forward(), the batched prompt
before the prompt loop, the routing record of every processed token and the
report at exit; and forward()'s own attention half copied into a function of
its own for the batched prompt.  The Makefile beside this file compiles the copy against
librbt_moe.so into _build/rabbit2_cuda.  Each edit is anchored on one engine
line and fails loudly if that line is missing or not unique.
"""
import sys

FORWARD = "static int forward(Model *m, State *s, int token, int pos, int32_t *routing_out) {"

INSERTIONS = [
    # (anchor line, where: before / after / replace, text)
    (FORWARD, "before", '#include "rbt_engine_hook.h"\n\n'),
    (FORWARD, "after",
     "    {\n"
     "        int f_ = rbt_engine_forward(m, s, token, pos, routing_out);\n"
     "        if (f_ < 0) return 0;\n"
     "        if (f_) return 1;\n"
     "    }\n"),
    ("        /* ---- MoE feed-forward ---- */", "after",
     "        {\n"
     "            int g_ = rbt_engine_moe(m, l, s->x, routing_out + (size_t)l * c->top_k);\n"
     "            if (g_ < 0) return 0;\n"
     "            if (g_) continue;\n"
     "        }\n"),
    ('        else if (!strcmp(argv[i], "--kernel") && i + 1 < argc) kernel = argv[++i];', "before",
     '        else if (!strcmp(argv[i], "--device") && i + 1 < argc) rbt_engine_device = argv[++i];\n'
     '        else if (!strcmp(argv[i], "--prefill") && i + 1 < argc) rbt_engine_prefill_mode = argv[++i];\n'
     '        else if (!strcmp(argv[i], "--offload") && i + 1 < argc) rbt_engine_offload = argv[++i];\n'
     '        else if (!strcmp(argv[i], "--routing-trace") && i + 1 < argc) rbt_engine_trace_path = argv[++i];\n'
     '        else if (!strcmp(argv[i], "--ep") && i + 1 < argc) rbt_engine_ep_arg = argv[++i];\n'),
    ("    if (!load_model(&m, argv[1])) return 1;", "after",
     "    if (!rbt_engine_init(&m)) return 1;\n"),
    ("    double t0 = now_sec();", "after",
     "    const int rbt_pre_ = rbt_engine_prefill(&m, &s, tokens, nt, routing, fl, fr);\n"
     "    if (rbt_pre_ < 0) {\n"
     "        if (fl) { fclose(fl); fclose(fr); }\n"
     "        return 1;\n"
     "    }\n"),
    ("    for (int i = 0; i < nt; i++) {", "replace",
     "    for (int i = rbt_pre_ ? nt : 0; i < nt; i++) {\n"),
    # the routing of every token forward() processed: prompt tokens, then generated ones
    ("        if (fl) {", "before", "        rbt_engine_record(&m, routing);\n"),
    ("            int next = sample_logits(s.logits, c->vocab, temperature, top_k_sample, top_p, &rng, sample_idx, "
     "sample_prob);", "before", "            if (g > 0) rbt_engine_record(&m, routing);\n"),
    ("    if (m.cache.file) {", "before", "    rbt_engine_report(&m);\n"),
]

# The engine's own attention half of a layer, hoisted out of forward() into a
# function of its own (written into the patched copy, from the engine's own lines):
# the batched prompt runs it for every prompt token of a layer before the layer's
# one MoE call.  Its locals are forward()'s prologue, verbatim.
HOIST_PROLOGUE_END = "    /* embedding row */"
HOIST_BEGIN = "        /* ---- attention ---- */"
HOIST_END = "        /* ---- MoE feed-forward ---- */"


def _index(lines, anchor):
    hits = [i for i, ln in enumerate(lines) if ln.rstrip("\n") == anchor]
    if len(hits) != 1:
        raise SystemExit(f"anchor found {len(hits)} times: {anchor!r}")
    return hits[0]


def hoisted_attention(lines) -> str:
    f = _index(lines, FORWARD)
    prologue = lines[f + 1:_index(lines, HOIST_PROLOGUE_END)]
    body = lines[_index(lines, HOIST_BEGIN):_index(lines, HOIST_END)]
    return ("/* forward()'s attention half of layer l for the token at position pos, on s->x\n"
            "   (copied from forward() by patch_engine.py) */\n"
            "#pragma GCC diagnostic push\n"
            "#pragma GCC diagnostic ignored \"-Wunused-variable\"\n"
            "static void rbt_engine_attention_block(Model *m, State *s, int l, int pos) {\n"
            + "".join(prologue) + "    const LayerOff *ly = &m->layers[l];\n" + "".join(body) + "}\n"
            "#pragma GCC diagnostic pop\n\n")


def patch(src: str) -> str:
    lines = src.splitlines(keepends=True)
    hoist = hoisted_attention(lines)
    for anchor, where, text in INSERTIONS:
        i = _index(lines, anchor)
        if where == "replace":
            lines[i] = text
        else:
            lines.insert(i if where == "before" else i + 1, text)
    lines.insert(_index(lines, '#include "rbt_engine_hook.h"'), hoist)
    return "".join(lines)


if __name__ == "__main__":
    with open(sys.argv[1]) as f:
        out = patch(f.read())
    with open(sys.argv[2], "w") as f:
        f.write(out)
