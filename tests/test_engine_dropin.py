"""The unmodified reference engine running on this library.

oracle/_ref/libtgai_engine_bridge.so is src/tgai_engine.c compiled with
TG_ENGINE_HAS_CUDA_BRIDGE and linked against libtgkv.so in place of the
reference's cuda/tgai_cuda_bridge.c + cuda/tgai_cuda.cu (oracle/Makefile).  A
child process (tests/engine_dropin_run.py) loads a seeded .TG model with the
engine's own tg_load and runs tg_forward over the script of
tests/fwd_model.py; the logits are compared with tests/golden/forward.npz,
which the engine built without the seam produced on the CPU.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import fwd_model as FM
from conftest import GOLDEN, ROOT

BRIDGE_SO = os.path.join(ROOT, "oracle", "_ref", "libtgai_engine_bridge.so")
RUNNER = os.path.join(ROOT, "tests", "engine_dropin_run.py")


def run_engine(tmp_path, name, use_gpu):
    if not os.path.exists(BRIDGE_SO):
        pytest.skip("oracle/_ref/libtgai_engine_bridge.so not built")
    cfg = FM.CONFIGS[name]
    model = tmp_path / f"{name}.TG"
    FM.write_tg(str(model), cfg, FM.weights(cfg, FM.SEEDS[name]))
    out = tmp_path / "out.npz"
    env = dict(os.environ)
    env.pop("TGAI_USE_GPU", None)
    if use_gpu:
        env["TGAI_USE_GPU"] = "1"
    r = subprocess.run([sys.executable, RUNNER, name, str(model), str(out)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    z = np.load(out)
    return z["logits"], str(z["reason"]), int(z["calls"]), int(z["fallbacks"])


def test_engine_with_seam_off_keeps_its_cpu_path(tmp_path):
    """Without TGAI_USE_GPU the engine's init leaves the model on the CPU and
    its logits are the golden ones bit for bit: the seam changes nothing."""
    lg, reason, calls, falls = run_engine(tmp_path, "moe", use_gpu=False)
    gold = np.load(os.path.join(GOLDEN, "forward.npz"))["moe_logits"]
    assert "TGAI_USE_GPU" in reason
    assert calls == 0 and falls == 0
    assert np.array_equal(lg, gold)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(FM.CONFIGS))
def test_engine_runs_on_the_gpu_forward(tmp_path, name):
    lg, reason, calls, falls = run_engine(tmp_path, name, use_gpu=True)
    gold = np.load(os.path.join(GOLDEN, "forward.npz"))[f"{name}_logits"]
    assert reason.startswith("TAKEN OVER"), reason
    assert calls == len(gold) and falls == 0
    err = float(np.max(np.abs(lg - gold).max(1) / np.abs(gold).max(1)))
    assert err < 1e-4, err
