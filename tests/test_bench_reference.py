"""The reference arm of ``bench.py`` (the oracle port on the host CPU) runs end to end
and prints the contract line.  The block forwards themselves are replaced by stubs here so
the test takes seconds; everything around it (imports, the workload's voxel set and
geometry, the line's keys) is the real code path."""
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_contract_line(monkeypatch, capsys):
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import model as om
    monkeypatch.setattr(om, "block_forward", lambda *a, **k: None)
    monkeypatch.setattr(om, "block_forward_1tok", lambda *a, **k: None)

    class Args:
        steps, warmup, gpus = 1, 0, 1

    monkeypatch.delenv("RANK", raising=False)
    # the arm must register the package itself (other tests register it for the session)
    monkeypatch.delitem(sys.modules, "vdit", raising=False)
    bench.run_reference(Args())
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "voxel-tokens/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["higher_is_better"] is True and line["config"]["seq_len"] == 16384
    # one timed step reaches the first block kind only; the other three are timed once at the end
    assert sorted(line["block_seconds"]) == sorted(bench.CPU_BLOCK_KINDS)
