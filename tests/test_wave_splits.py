"""The split-K rule of the weight-gradient and LSTM products (wave_splits in
nn_in_trading_b200/csrc/wgrad.cuh), compiled for the host by nvcc and run on the CPU: the chosen
split count keeps its work items within 3 % of the best whole-wave efficiency of one, two or three
waves of the 148 SMs, is the fewest that does, never exceeds its cap, and is 1 once the output tiles
alone fill the SMs.  Plus the counts of the shapes the benchmarks run."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
SMS = 148

pytestmark = pytest.mark.skipif(not (os.path.exists(NVCC) or shutil.which("nvcc")), reason="no nvcc")


@pytest.fixture(scope="module")
def splits(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("wave") / "wave_splits_check")
    src = os.path.join(ROOT, "tests", "cpp", "wave_splits_check.cu")
    r = subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "--expt-relaxed-constexpr",
                        src, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

    def run(pairs):
        text = "".join(f"{t} {c}\n" for t, c in pairs)
        out = subprocess.run([exe], input=text, capture_output=True, text=True, check=True, timeout=60).stdout
        return {(int(a), int(b)): int(s) for a, b, s in (line.split() for line in out.splitlines())}
    return run


def efficiency(tiles, s):
    items = tiles * s
    return items / (SMS * -(-items // SMS))


def test_rule_properties_over_a_sweep(splits):
    pairs = [(t, c) for t in range(1, 201) for c in (1, 2, 4, 8, 16, 64, 4096)]
    got = splits(pairs)
    for (t, c), s in got.items():
        if t >= SMS:
            assert s == 1, (t, c, s)
            continue
        assert 1 <= s <= max(c, 1), (t, c, s)
        cands = [min(max(w * SMS // t, 1), max(c, 1)) for w in (1, 2, 3)]
        best = max(efficiency(t, x) for x in cands)
        assert efficiency(t, s) >= best - 0.03 - 1e-12, (t, c, s)
        assert s == min(x for x in cands if efficiency(t, x) >= best - 0.03 - 1e-12), (t, c, s)


def test_counts_of_the_benchmark_shapes(splits):
    cases = {
        (1, 4096): 148,  # one 128 x 128 tile over a million rows: one full wave
        (24, 8): 6,      # LSTM weight gradient of layer 1, 1024 x 320 over 1024 series: one wave of 144 items
        (32, 8): 4,      # LSTM weight gradient of layer 2, 1024 x 512: 128 items, as efficient as 256
        (40, 4): 3,      # LSTM gate product of layer 2, 1024 x 260 in 128 x 64 tiles, K = 512
        (4, 16): 16,     # SAC critic head, 1 x 512 over 4096 transitions: capped at K / 256
        (6, 120): 24,    # encoder Q/K/V weight gradient, 768 x 64 over 30,720 rows (batch 256)
        (148, 64): 1,
        (480, 64): 1,
    }
    got = splits(list(cases))
    assert got == cases
