"""bench.py's reference arm on the CPU (no GPU needed): the reference's path on the host cores for
a config, printed as one JSON line with the contract's keys. For the attention config the timed
code is the reference's own compiled onpu_attn_step_bf16 when oracle/_ref was built."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parents[1]


def _reference_line(config):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", config, "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("config,unit", [("attn", "GB/s"), ("gemv", "GB/s"), ("qwen2.5-32b", "tokens/s")])
def test_reference_arm_prints_one_contract_line(config, unit):
    d = _reference_line(config)
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    for key in ("metric", "n_gpus", "steps", "warmup", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    if config == "qwen2.5-32b":            # the default config: the same config dict as our arm's line
        sys.path.insert(0, str(ROOT))
        import bench
        assert d["config"] == bench.tp_config(1, 64, 1) and d["scaling"] == "strong"
    if config == "attn":
        assert d["config"]["context"] == 4096
        assert d["cpu_baseline"]["kind"] == ("reference" if O.ref_lib() is not None else "port")

