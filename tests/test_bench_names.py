"""bench.py's two arms describe the same workload: the reference arm's policy
names (it loads no engine code) equal the engine arm's sweep, in order."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def test_reference_arm_names_the_engine_sweep():
    import bench
    import drift_b200 as d

    assert [p.name for p in bench.sweep_policies(d)] == bench.SWEEP_NAMES
