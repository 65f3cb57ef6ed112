"""The CUDA-core attention kernel (aspire_attn_gather_kernel) takes the rows
that the routing thresholds keep off the tcgen05 kernel.  By default every row
is routed to tcgen05, so this test reruns the attention parity tests in a
child process whose thresholds send narrow rows (packed query tile <= 4 rows,
context below 10^9 tokens) to the CUDA-core kernel, and with tcgen05 off."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("env", [
    {"ASPIRE_B200_TC_MIN_ROWS": "5", "ASPIRE_B200_TC_MIN_KV": "1000000000"},
    {"ASPIRE_B200_DISABLE_TC": "1"},
], ids=["narrow_rows_on_cuda_cores", "tcgen05_off"])
def test_attention_parity_on_cuda_core_route(cuda_device, env):
    child_env = dict(os.environ, ASPIRE_B200_NO_BUILD="1", **env)
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        str(ROOT / "tests" / "test_attention_gpu.py")],
                       cwd=ROOT, env=child_env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
