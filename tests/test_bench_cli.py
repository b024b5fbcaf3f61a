"""bench.py's reference arm runs on CPU and keeps the JSON contract, for both
code widths.  The arm times the reference's own pure-PyTorch optimizer
(baseline/mdqbock_newhook.py, byte-compiled into oracle/_ref by the build) and
falls back to the C restatement of the reference kernel when that module was
not built."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("bits", [4, 8])
def test_reference_arm_json_line(bits):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "3", "--warmup", "3", "--bits", str(bits)],
                         capture_output=True, text=True, timeout=300, cwd=REPO, check=True)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "Gparams/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["config"]["bits"] == bits
    base = line["cpu_baseline"]
    ref_built = os.path.isfile(os.path.join(REPO, "oracle", "_ref", "mdqbock_newhook.pycode"))
    assert base["kind"] == ("reference" if ref_built else "port") and base["cores"] >= 1
    if ref_built:
        assert "mdqbock_newhook" in base["sample"] and "8]-bit" in base["sample"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_warmup_below_three_is_refused():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--warmup", "2"],
                       capture_output=True, text=True, timeout=120, cwd=REPO)
    assert r.returncode != 0 and "warmup" in r.stderr
