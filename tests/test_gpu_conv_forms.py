"""Both forms of the conv layer kernel stay bit-exact against the oracle.  Layers without
needs_tail run the queue form (conv_queue) by default, so the chunked form (conv_fused) would be
exercised only by tail layers; here the layer and configuration parity suites run once more in a
child process with SALT_CONV_FORM=chunked (the library reads it once per process)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_chunked_form_passes_the_parity_suites():
    env = dict(os.environ, SALT_CONV_FORM="chunked")
    suites = [os.path.join(HERE, "test_gpu_layer_parity.py"),
              os.path.join(HERE, "test_gpu_configs.py")]
    r = subprocess.run([sys.executable, "-m", "pytest", *suites, "-x", "-q", "-m", "gpu",
                        "-p", "no:cacheprovider"],
                       cwd=os.path.dirname(HERE), env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
