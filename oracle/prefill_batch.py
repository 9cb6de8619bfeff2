"""The prefill caller change, applied to the reference engine's sources.

In the engine's batch prefill the out_proj of a DeltaNet layer
(qwen35-c/src/q35_deltanet.c:491-499) and the o_proj of a GQA layer
(qwen35-c/src/q35_attn.c:262, reached per token from :308-318) are called
once per token through q35_mm_fp8, so each re-streams its 31.5 MB weight for
every token.  This script rewrites those two call sites so that each layer
makes ONE q35_mm_fp8_batch call over all its tokens -- the change a
maintainer would make to use the batched entry point (the GPU library's
tensor-core GEMM for 128 tokens or more):

* DeltaNet: the gated RMS norm runs on every token's output rows in place
  (all_o is not read again), then one q35_mm_fp8_batch(w_out, ..., L, all_o, y);
* GQA: a file-scope switch makes attn_token_core leave its gated attention
  output (q_heads * head_dim values) in `out` instead of projecting it; the
  batch branch collects every token's into one buffer and then makes one
  q35_mm_fp8_batch(wo, ..., nt, all_sa, out).  The single-token path is
  unchanged.

Behaviour kept: the results are bit-identical to the per-token calls for
batches the library runs on its decode GEMV (fewer than 16 tokens) and within
the library's batch contracts above that.  On an attention error part-way
through a batch (a full KV cache) the patched engine writes no output rows,
where the original wrote those of the tokens before the failing one.

The edits are given as line ranges of the reference files, pinned by their
sha256 so a changed tree is refused rather than patched blindly; the
replacement text is this project's.  Usage (oracle/Makefile `engine-batched`):

    python prefill_batch.py <qwen35-c dir> <output dir>

writes the patched q35_deltanet.c and q35_attn.c into <output dir>.
"""
from __future__ import annotations

import hashlib
import os
import sys

PINS = {
    "src/q35_deltanet.c": "b8684d5d7a5bce876e4da0bf497105ffd257edb127f5d91561ecc5b6ad97e11d",
    "src/q35_attn.c": "b0082b541200eca2669e7328eefa12b5ecb850b8246d7c17de9f122bd52b89a2",
}

# (file, first line, last line, replacement); lines are 1-based and inclusive;
# last = first - 1 inserts before `first`.  Applied bottom-up per file.
EDITS = [
    ("src/q35_deltanet.c", 491, 499, """\
        /* gated RMS norm of every token's output rows, in place, then one
         * batched out_proj over all L tokens */
        for (size_t t = 0; t < L; t++)
            for (h = 0; h < Hv; h++)
                dn_rmsnorm_gated(all_o + t * V + (size_t)h * dv,
                                 all_zq + t * V + (size_t)h * dv,
                                 layer->gate_norm_w, dv, norm_eps);
        q35_mm_fp8_batch(layer->w_out, layer->sc_out, H, V, (uint32_t)L, all_o, y);
"""),
    ("src/q35_attn.c", 173, 172, """\
/* Set by the batched prefill below: attn_token_core then leaves the gated
 * attention output (q_heads * head_dim values) in `out` and the caller
 * projects every token's with one q35_mm_fp8_batch. */
static int attn_oproj_deferred = 0;

"""),
    ("src/q35_attn.c", 262, 262, """\
    if (attn_oproj_deferred)
        memcpy(out, sa, (size_t)qh * hd * sizeof(float));
    else
        q35_mm_fp8(w->wo, w->wo_sc, cfg->hidden, qh * hd, sa, out);
"""),
    ("src/q35_attn.c", 308, 319, """\
        float *all_sa = (float *)malloc((size_t)nt * qh * hd * sizeof(float));
        if (!all_sa) {
            free(all_sq); free(all_sk); free(all_sv);
            return Q35_ATTN_ERR_ARG;
        }
        attn_oproj_deferred = 1;
        for (uint32_t t = 0; t < nt; t++) {
            /* core modifies its k copy (norm, rope) in place */
            memcpy(sk, all_sk + (size_t)t * krows, (size_t)krows * sizeof(float));
            rc = attn_token_core(cfg, w, cache, all_sq + (size_t)t * qrows, sk,
                                 all_sv + (size_t)t * krows,
                                 all_sa + (size_t)t * qh * hd, sa, sg, sc);
            if (rc) break;
        }
        attn_oproj_deferred = 0;
        if (!rc) q35_mm_fp8_batch(w->wo, w->wo_sc, cfg->hidden, qh * hd, nt, all_sa, out);
        free(all_sa); free(all_sq); free(all_sk); free(all_sv);
"""),
]


def sha256(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def patch(ref: str, out: str) -> list[str]:
    os.makedirs(out, exist_ok=True)
    written = []
    for rel, pin in PINS.items():
        src = os.path.join(ref, rel)
        got = sha256(src)
        if got != pin:
            raise SystemExit(f"{src}: sha256 {got} is not the pinned {pin}; refusing to patch")
        with open(src) as f:
            lines = f.read().split("\n")
        for _, first, last, text in sorted((e for e in EDITS if e[0] == rel), key=lambda e: -e[1]):
            lines[first - 1:last] = text.rstrip("\n").split("\n")
        dst = os.path.join(out, os.path.basename(rel))
        with open(dst, "w") as f:
            f.write("\n".join(lines))
        written.append(dst)
    return written


if __name__ == "__main__":
    if len(sys.argv) != 3:
        raise SystemExit(__doc__)
    for p in patch(sys.argv[1], sys.argv[2]):
        print(p)
