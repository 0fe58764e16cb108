"""Every decode attention kernel, forced by VOX_CUDA_ATTN in a child process
(the choice is read once per process): v3 (one 64-key split per CTA), v4
(pipelined 32-key tiles), v4's deep variant (3 tile buffers) and v5 (keys
streamed into registers; 8-warp CTAs for one or two rows, 4-warp CTAs for
more).  Each runs the stand-alone attention against the reference's golden
vectors (L = 1 .. 8192, wrapped rings), the batched step against single
streams and the oracle, and the prefills (many rows of one sequence in one
launch, fresh keys) against their references (voxtral_kernels.c:412-482)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
SELECT = ("attention_decode_matches or batched_step_matches_single or prefill_batch_matches "
          "or tc_prefill_across or tc_prefill_matches")


@pytest.mark.parametrize("variant", ["v3", "v4", "deep", "v5"])
def test_attention_variant_matches_reference(variant):
    env = dict(os.environ, VOX_CUDA_ATTN=variant)
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(HERE, "test_gpu_decode.py"), "-q", "-x",
                        "-m", "gpu", "-p", "no:cacheprovider", "-k", SELECT],
                       env=env, capture_output=True, text=True, timeout=900, cwd=os.path.dirname(HERE))
    tail = (r.stdout[-3000:] + r.stderr[-2000:])
    assert r.returncode == 0, tail
    assert " passed" in r.stdout and " failed" not in r.stdout, tail
