"""Build recipe: the RABBIT2 engine with its MoE block (or its whole forward) on the GPU.

    python rabbit2_b200/engine/patch_engine.py <rabbit2.c> <out.c>

Writes a copy of the engine source (rabbit2/src/rabbit2.c) with these edits and
nothing else changed: the include of rbt_engine_hook.h, its CLI flags, its init
call, the whole-forward and MoE-block calls in forward(), and the batched prompt
before the prompt loop.  The Makefile beside this file compiles the copy against
librbt_moe.so into _build/rabbit2_cuda.  Each edit is anchored on one engine
line and fails loudly if that line is missing or not unique.
"""
import sys

INSERTIONS = [
    # (anchor line, where: before / after / replace, text)
    ("static int forward(Model *m, State *s, int token, int pos, int32_t *routing_out) {", "before",
     '#include "rbt_engine_hook.h"\n\n'),
    ("static int forward(Model *m, State *s, int token, int pos, int32_t *routing_out) {", "after",
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
     '        else if (!strcmp(argv[i], "--offload") && i + 1 < argc) rbt_engine_offload = argv[++i];\n'),
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
]


def patch(src: str) -> str:
    lines = src.splitlines(keepends=True)
    for anchor, where, text in INSERTIONS:
        hits = [i for i, ln in enumerate(lines) if ln.rstrip("\n") == anchor]
        if len(hits) != 1:
            raise SystemExit(f"anchor found {len(hits)} times: {anchor!r}")
        i = hits[0]
        if where == "replace":
            lines[i] = text
        else:
            lines.insert(i if where == "before" else i + 1, text)
    return "".join(lines)


if __name__ == "__main__":
    with open(sys.argv[1]) as f:
        out = patch(f.read())
    with open(sys.argv[2], "w") as f:
        f.write(out)
