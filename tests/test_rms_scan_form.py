"""Every RMS form, selected with TILER_RMS_FORM (read once per process) --
warp-per-row (rms_scan.cu, "scan"), chunk-streamed (rms_stream.cu, "stream"),
wave ("wave") -- held to the same parity tests the default selection passes:
the RMS f32 / bf16 oracle cases at full and ragged sizes, the fold stress rows
(ties, binade crossings, tiny and overflowing sums, NaN / inf) and the fused
quantize, run in a child process with the form selected."""
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("form", ["scan", "stream", "wave"])
def test_rms_form_passes_the_rms_parity_tests(form):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    env = dict(os.environ, TILER_RMS_FORM=form)
    sel = "rms_norm_f32_matches or rms_norm_bf16_matches or fold_stress or quantize_fusion"
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(ROOT, "tests", "test_gpu_parity.py"), "-k", sel],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
