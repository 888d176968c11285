"""Apply the GPU routing edit to charsiu's own decode loop. TEST INFRASTRUCTURE.

    python oracle/route_llama.py REF/src/llama.c OUT.c

Writes OUT.c: the reference's src/llama.c with the five insertions a
maintainer makes to route every projection and the head through the GPU
layer (include/charsiu_gpu.h) when CHARSIU_GPU is set -- the edit that
INTEGRATION.md describes, applied mechanically so that a test can build and run
charsiu's unmodified llama_forward / matvec_pair / matvec_again around it.
oracle/Makefile runs this into a temporary file, compiles it and deletes it;
nothing of the reference is kept in this repository.

Each insertion goes at an anchor that must occur exactly once in the file (so a
changed reference fails here, loudly, instead of building something else):

  1. after the charsiu_llm.h include: the GPU header and the layer handle;
  2. in llama_state_new, before the pool starts: the open (src/llama.c:568-582
     is the NPU's twin);
  3. at the top of matvec_pair, after the activation is quantised
     (src/llama.c:215-248): q/k/v or gate/up as one group call;
  4. at the top of matvec_again (src/llama.c:250-312): one projection;
  5. in llama_state_free, beside the NPU report (src/llama.c:671-673): the
     report and the close.

A -1 from the layer falls through to the CPU code below each insertion, as an
NPU refusal does.
"""
from __future__ import annotations

import re
import sys

# the layer handle lives at file scope: one decode state at a time, which is
# how charsiu_run and the tests use the loop
HEADER = """
#include "charsiu_gpu.h"

/* CHARSIU_GPU=1: every q8_0 / q4_0 projection and the head on the GPU */
static struct charsiu_gpu *gpu_layer;
"""

OPEN = """\tif (getenv("CHARSIU_GPU") && !gpu_layer) {
\t\tunsigned gwide = m->n_embd > m->n_ff ? m->n_embd : m->n_ff;

\t\tgpu_layer = charsiu_gpu_open(gwide, m->n_vocab > gwide ? m->n_vocab : gwide,
\t\t\t\t\t     s->npu_cap);
\t\tfprintf(stderr, gpu_layer ? "charsiu: GPU open\\n"
\t\t\t\t\t  : "charsiu: no GPU; staying on the CPU\\n");
\t}

"""

GROUP = """\tif (gpu_layer && s->act.quantised && !getenv("CHARSIU_GPU_NOGROUP")) {
\t\tint gids[3];
\t\tunsigned gi;

\t\tfor (gi = 0; gi < n; gi++)
\t\t\tif ((gids[gi] = charsiu_gpu_add(gpu_layer, w[gi])) < 0)
\t\t\t\tbreak;
\t\tif (gi == n && !charsiu_gpu_matvec_group(gpu_layer, gids, n, &s->act, y))
\t\t\treturn;
\t}
"""

SINGLE = """\tif (gpu_layer && a->quantised) {
\t\tint gid = charsiu_gpu_add(gpu_layer, w);

\t\tif (gid >= 0 && !charsiu_gpu_matvec(gpu_layer, gid, a, y))
\t\t\treturn;
\t}
"""

CLOSE = """\tif (gpu_layer) {
\t\tif (getenv("CHARSIU_GPU_REPORT"))
\t\t\tcharsiu_gpu_report(gpu_layer);
\t\tcharsiu_gpu_close(gpu_layer);
\t\tgpu_layer = NULL;
\t}
"""

# (anchor regex, text, where: "after" the match or "before" it)
EDITS = [
    (r'#include "charsiu_llm\.h"\n', HEADER, "after"),
    (r"\n\tpool_start\(0\);\n\treturn s;\n", OPEN, "before_body"),
    (r"\tcharsiu_act_set\(&s->act, x, \(int\)wa->ne\[0\]\);\n", GROUP, "after"),
    (r"static void matvec_again\(struct llama_state \*s, const struct gguf_tensor \*w,\n"
     r"\s*float \*y\)\n\{\n\tstruct charsiu_act \*a = &s->act;\n"
     r"\tconst struct npu_tensor \*nt = NULL;\n", SINGLE, "after"),
    (r"\tllama_stages_report\(\);\n", CLOSE, "before"),
]


def route(src: str) -> str:
    for pat, text, where in EDITS:
        hits = list(re.finditer(pat, src))
        if len(hits) != 1:
            raise SystemExit(f"route_llama: anchor {pat!r} found {len(hits)} times, want 1")
        h = hits[0]
        if where == "after":
            src = src[:h.end()] + text + src[h.end():]
        elif where == "before":
            src = src[:h.start()] + text + src[h.start():]
        else:   # before the matched statements, after their leading newline
            src = src[:h.start() + 1] + text + src[h.start() + 1:]
    return src


def main() -> None:
    if len(sys.argv) != 3:
        raise SystemExit(__doc__)
    with open(sys.argv[1]) as f:
        out = route(f.read())
    with open(sys.argv[2], "w") as f:
        f.write(out)


if __name__ == "__main__":
    main()
