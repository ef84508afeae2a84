"""CPU checks of the roofline figures ``bench.py`` reports: the algorithmic bytes one Euler step must
stream from HBM at the BASELINE configs[1] shapes, and the ncu traffic figure read from the committed
expert-kernel profile summary."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from reki_megakernel_b200.synthetic import ExpertDims  # noqa: E402


def test_algorithmic_bytes_per_euler_step():
    d = ExpertDims()
    mods_row = 2 * d.MODW                       # one bf16 modulation row: 70,656 values
    assert mods_row == 141_312
    per_step = bench.algorithmic_bytes_per_step(d, mods_row)
    # bf16 weights 212,336,640 + fp32 in/out projections 196,608 + norm weights 3,840 + one row
    assert per_step == 212_336_640 + 196_608 + 3_840 + 141_312 == 212_678_400
    assert 9 * per_step == 1_914_105_600        # one launch = Euler steps 2..10


def test_traffic_figure_is_tied_to_the_kernel_sources_it_was_captured_from():
    """The ncu summary records the sha of the kernel sources it profiled; bench.py reports its
    traffic figure only while the sources are the same, and says why when they are not."""
    t, src = bench.traffic_from_profile()
    text = (ROOT / "profiles" / "expert_kernel_full.md").read_text()
    recorded = [ln.split(":", 1)[1].split()[0] for ln in text.splitlines() if ln.startswith("kernel_source_sha16:")]
    if recorded and recorded[0] == bench.kernel_source_sha():
        assert t is not None and "ncu capture" in src
        # ncu's DRAM bytes of one launch: within 1 % of the algorithmic bytes (no re-reads)
        assert abs(t / 1_914_105_600 - 1.0) < 0.01
    else:
        assert t is None and "other kernel sources" in src
