#!/usr/bin/env python3
"""Write the `make cuda` source tree: the reference's C sources copied from
their tree, with the USE_CUDA hooks inserted where the `make mps` build calls
voxtral_metal.h.

    python3 integration/apply_cuda.py <reference dir> <output dir>

Every hook is a few lines of this project's own code, placed by an anchor: a
line of the reference that must occur exactly once (or the first line ending in
"{" after it, for a function's opening).  A missing or repeated anchor stops the
build with a message, so a changed reference tree is noticed rather than
patched in the wrong place.  The reference tree itself is only read.

Hook sites (reference file:line):
  voxtral.h:201            vox_ctx_t gets the device handles; the host glue's
                           prototypes follow the header (voxtral_cuda_host.h)
  voxtral_kernels.c:197-264  vox_linear_nobias_bf16 / vox_linear_bf16 /
                           vox_matmul_t_bf16 -> vox_cuda_sgemm_bf16
  voxtral_decoder.c:233    vox_decoder_prefill -> the device prefill
  voxtral_decoder.c:401    vox_decoder_forward -> the device decode step
  voxtral_encoder.c:452    vox_encoder_forward_incremental -> the device encoder
  voxtral_encoder.c:642    vox_adapter_forward -> the device adapter
  voxtral.c:243-246        vox_load ends by uploading the model (attach)
  voxtral.c:253            vox_free releases the device copies (detach)
  voxtral.c:1344-1350      vox_set_delay rewrites the device's ada scale
  main.c:162-164, 283-285  vox_cuda_init / vox_cuda_shutdown
"""
from __future__ import annotations

import os
import shutil
import sys

SOURCES = ["voxtral.c", "voxtral_kernels.c", "voxtral_audio.c", "voxtral_encoder.c",
           "voxtral_decoder.c", "voxtral_tokenizer.c", "voxtral_safetensors.c", "main.c",
           "voxtral.h", "voxtral_kernels.h", "voxtral_audio.h", "voxtral_tokenizer.h",
           "voxtral_safetensors.h", "voxtral_metal.h"]


class AnchorError(RuntimeError):
    pass


def find_once(lines, text, start=0, fname=""):
    hits = [i for i in range(start, len(lines)) if lines[i].rstrip("\n") == text]
    if len(hits) != 1:
        raise AnchorError(f"{fname}: anchor {text!r} found {len(hits)} times (want 1)")
    return hits[0]


def find_first(lines, text, start, fname):
    for i in range(start, len(lines)):
        if lines[i].rstrip("\n") == text:
            return i
    raise AnchorError(f"{fname}: anchor {text!r} not found after line {start + 1}")


def opening_brace(lines, sig_line, fname):
    """Index of the first line at or after sig_line that ends with '{'."""
    for i in range(sig_line, min(sig_line + 6, len(lines))):
        if lines[i].rstrip().endswith("{"):
            return i
    raise AnchorError(f"{fname}: no opening brace after line {sig_line + 1}")


def block(*code):
    return "".join(c + "\n" for c in code)


def hook_function_entry(lines, fname, signature_start, code):
    """Insert `code` right after the opening brace of the function whose
    signature starts with the line `signature_start`."""
    i = find_once(lines, signature_start, 0, fname)
    j = opening_brace(lines, i, fname)
    lines.insert(j + 1, code)


SGEMM_HOOK = (
    "#ifdef USE_CUDA\n"
    "    if (vox_cuda_available() &&\n"
    "        vox_cuda_sgemm_bf16({M}, {N}, {K}, {A}, {B}, {bias}, {C}) == VOX_CUDA_OK)\n"
    "        return;\n"
    "#endif\n")


def patch_voxtral_h(lines, f):
    i = find_once(lines, "} vox_ctx_t;", 0, f)
    lines.insert(i, block(
        "#ifdef USE_CUDA",
        "    /* device copies made by vox_cuda_host_attach (voxtral_cuda_host.h) */",
        "    void *cuda_dec;          /* vox_cuda_decoder *: resident decoder weights */",
        "    void *cuda_state;        /* vox_cuda_dec_state *: the decoder KV ring */",
        "    void *cuda_enc;          /* vox_cuda_encoder *: encoder + adapter weights */",
        "    void *cuda_enc_state;    /* vox_cuda_enc_state *: the encoder KV ring */",
        "#endif"))
    i = find_once(lines, "#endif /* VOXTRAL_H */", 0, f)
    lines.insert(i, block("#ifdef USE_CUDA", '#include "voxtral_cuda_host.h"', "#endif"))


def patch_kernels(lines, f):
    i = find_once(lines, '#include "voxtral_kernels.h"', 0, f)
    lines.insert(i + 1, block("#ifdef USE_CUDA", '#include "voxtral_cuda.h"', "#endif"))
    hook_function_entry(lines, f, "void vox_linear_nobias_bf16(float *y, const float *x, const uint16_t *W_bf16,",
                        SGEMM_HOOK.format(M="seq_len", N="out_dim", K="in_dim", A="x", B="W_bf16",
                                          bias="NULL", C="y"))
    hook_function_entry(lines, f, "void vox_linear_bf16(float *y, const float *x, const uint16_t *W_bf16,",
                        SGEMM_HOOK.format(M="seq_len", N="out_dim", K="in_dim", A="x", B="W_bf16",
                                          bias="b", C="y"))
    hook_function_entry(lines, f, "void vox_matmul_t_bf16(float *C, const float *A, const uint16_t *B_bf16,",
                        SGEMM_HOOK.format(M="M", N="N", K="K", A="A", B="B_bf16", bias="NULL", C="C"))


def patch_decoder(lines, f):
    hook_function_entry(lines, f,
                        "void vox_decoder_prefill(vox_ctx_t *ctx, const float *input_embeds, int seq_len) {",
                        block("#ifdef USE_CUDA",
                              "    if (ctx->cuda_state) {   /* no CPU fallback: a failure is reported */",
                              "        vox_cuda_host_decoder_prefill(ctx, input_embeds, seq_len);",
                              "        return;",
                              "    }",
                              "#endif"))
    hook_function_entry(lines, f,
                        "int vox_decoder_forward(vox_ctx_t *ctx, const float *input_embeds, float *logits) {",
                        block("#ifdef USE_CUDA",
                              "    if (ctx->cuda_state) return vox_cuda_host_decoder_forward(ctx, input_embeds, logits);",
                              "#endif"))


def patch_encoder(lines, f):
    hook_function_entry(lines, f, "float *vox_encoder_forward_incremental(vox_ctx_t *ctx, const float *x_new,",
                        block("#ifdef USE_CUDA",
                              "    if (ctx->cuda_enc_state)",
                              "        return vox_cuda_host_encoder_incremental(ctx, x_new, new_len, out_len);",
                              "#endif"))
    hook_function_entry(lines, f, "float *vox_adapter_forward(vox_ctx_t *ctx, const float *enc_out,",
                        block("#ifdef USE_CUDA",
                              "    if (ctx->cuda_enc_state)",
                              "        return vox_cuda_host_adapter_forward(ctx, enc_out, enc_seq_len, out_seq_len);",
                              "#endif"))


def patch_voxtral_c(lines, f):
    i = find_once(lines, 'vox_ctx_t *vox_load(const char *model_dir) {', 0, f)
    j = find_first(lines, '        fprintf(stderr, "Model loaded.\\n");', i, f)
    # before the `if (vox_verbose >= 1)` that prints "Model loaded."
    lines.insert(j - 1, block(
        "#ifdef USE_CUDA",
        "    /* upload the model once; the layer loops then run on the device */",
        "    if (vox_cuda_available() && vox_cuda_host_attach(ctx) != 0)",
        '        fprintf(stderr, "CUDA: model upload failed; the CPU path is used\\n");',
        "#endif"))
    i = find_once(lines, "void vox_free(vox_ctx_t *ctx) {", 0, f)
    j = find_first(lines, "    if (!ctx) return;", i, f)
    lines.insert(j + 1, block("#ifdef USE_CUDA", "    vox_cuda_host_detach(ctx);", "#endif"))
    i = find_once(lines, "void vox_set_delay(vox_ctx_t *ctx, int delay_ms) {", 0, f)
    j = find_first(lines, "    vox_update_time_conditioning(ctx);", i, f)
    lines.insert(j + 1, block("#ifdef USE_CUDA", "    vox_cuda_host_ada_changed(ctx);", "#endif"))


def patch_main(lines, f):
    i = find_once(lines, '#include "voxtral_audio.h"', 0, f)
    lines.insert(i + 1, block("#ifdef USE_CUDA", '#include "voxtral_cuda.h"', "#endif"))
    i = find_once(lines, "    vox_metal_init();", 0, f)
    j = find_first(lines, "#endif", i, f)
    lines.insert(j + 1, block(
        "#ifdef USE_CUDA",
        "    if (!vox_cuda_init()) fprintf(stderr, \"CUDA unavailable: %s\\n\", vox_cuda_last_error());",
        "#endif"))
    i = find_once(lines, "    vox_metal_shutdown();", 0, f)
    j = find_first(lines, "#endif", i, f)
    lines.insert(j + 1, block("#ifdef USE_CUDA", "    vox_cuda_shutdown();", "#endif"))


PATCHES = {
    "voxtral.h": patch_voxtral_h,
    "voxtral_kernels.c": patch_kernels,
    "voxtral_decoder.c": patch_decoder,
    "voxtral_encoder.c": patch_encoder,
    "voxtral.c": patch_voxtral_c,
    "main.c": patch_main,
}


def main(argv):
    if len(argv) != 3:
        print(__doc__)
        return 2
    ref, out = argv[1], argv[2]
    os.makedirs(out, exist_ok=True)
    for name in SOURCES:
        src = os.path.join(ref, name)
        if not os.path.exists(src):
            raise SystemExit(f"apply_cuda: {src} missing")
        dst = os.path.join(out, name)
        if name in PATCHES:
            with open(src) as fh:
                lines = fh.readlines()
            PATCHES[name](lines, name)
            with open(dst + ".tmp", "w") as fh:
                fh.writelines(lines)
            os.replace(dst + ".tmp", dst)
        else:
            shutil.copyfile(src, dst)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
