"""The `make cuda` recipe (integration/) on the CPU: the hook script refuses a
reference tree whose anchors moved, and the built CLI starts (its usage text)
without touching a GPU."""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INTEG = os.path.join(ROOT, "integration")
REF = os.environ.get("VOX_REFERENCE_DIR", "/root/reference")
sys.path.insert(0, INTEG)
import apply_cuda  # noqa: E402


def test_hooks_land_once_each(tmp_path):
    if not os.path.isdir(REF):
        pytest.skip("reference tree not present on this machine")
    out = tmp_path / "src"
    assert apply_cuda.main(["apply_cuda.py", REF, str(out)]) == 0
    text = {n: (out / n).read_text() for n in apply_cuda.PATCHES}
    assert text["voxtral_kernels.c"].count("vox_cuda_sgemm_bf16(") == 3
    assert "vox_cuda_host_decoder_forward" in text["voxtral_decoder.c"]
    assert "vox_cuda_host_decoder_prefill" in text["voxtral_decoder.c"]
    assert "vox_cuda_host_encoder_incremental" in text["voxtral_encoder.c"]
    assert "vox_cuda_host_adapter_forward" in text["voxtral_encoder.c"]
    assert text["voxtral.c"].count("vox_cuda_host_") == 3
    assert "vox_cuda_init()" in text["main.c"] and "vox_cuda_shutdown()" in text["main.c"]
    # every hook is compiled only for the cuda build
    for n, t in text.items():
        assert t.count("#ifdef USE_CUDA") >= 1, n


def test_a_moved_anchor_stops_the_build(tmp_path):
    if not os.path.isdir(REF):
        pytest.skip("reference tree not present on this machine")
    ref = tmp_path / "ref"
    shutil.copytree(REF, ref, ignore=shutil.ignore_patterns(".git", "*.o", "samples", "*.wav"))
    p = ref / "voxtral_decoder.c"
    p.write_text(p.read_text().replace(
        "int vox_decoder_forward(vox_ctx_t *ctx, const float *input_embeds, float *logits) {",
        "int vox_decoder_forward(vox_ctx_t *ctx, const float *embeds, float *logits) {"))
    with pytest.raises(apply_cuda.AnchorError):
        apply_cuda.main(["apply_cuda.py", str(ref), str(tmp_path / "out")])


def test_cuda_cli_starts():
    exe = os.path.join(INTEG, "_build", "voxtral")
    if not os.path.exists(exe):
        pytest.skip("integration not built (needs the reference tree)")
    r = subprocess.run([exe, "-h"], capture_output=True, text=True, timeout=60)
    assert "Usage" in r.stdout + r.stderr
