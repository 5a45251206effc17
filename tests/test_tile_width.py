"""The GEMM tile-width rule (`pick_tile_n` in csrc/gemm_sm100.cuh), on the host: 192-wide tiles
where N is a whole number of them and they need fewer waves x width, at deep K only when the
256-wide tiles do not fill one wave. Compiled with nvcc into a small host program; no GPU."""

import subprocess

import pytest

from conftest import REPO

PROGRAM = r"""
#include <cstdio>
#include "gemm_sm100.cuh"
int main() {
  const long long cases[][5] = {CASES};
  for (auto& c : cases)
    printf("%d\n", ppyb200::gemm::pick_tile_n(c[0], c[1], c[2], c[3], c[4]));
  return 0;
}
"""

# (m, n, k, rows per CTA pair, CTA pairs) -> width; GPT-2's layers at 4 and 32 sequences
CASES = [
    ((4096, 768, 3072, 256, 74), 192),   # proj, 4 sequences: 48 of 74 pairs busy with 256
    ((32768, 768, 3072, 256, 74), 256),  # proj, 32 sequences: deep K, several waves
    ((4096, 768, 768, 256, 74), 192),    # out projection, one wave either way, narrower
    ((32768, 768, 768, 256, 74), 192),   # out projection: 7 waves of 192 against 6 of 256
    ((4096, 2304, 768, 256, 74), 256),   # QKV: 2 waves of 256 against 3 of 192
    ((8192, 8192, 8192, 256, 74), 256),  # N not a multiple of 192
]


def test_tile_width_rule(tmp_path):
    from ppy_b200 import toolchain

    tool = toolchain.nvcc()
    if tool is None:
        pytest.skip("nvcc is not installed")
    source = tmp_path / "tile_width.cu"
    source.write_text(PROGRAM.replace(
        "CASES", ", ".join("{%d, %d, %d, %d, %d}" % c for c, _ in CASES)))
    binary = tmp_path / "tile_width"
    subprocess.run([tool, "-std=c++17", "--expt-relaxed-constexpr", "-diag-suppress", "177,550",
                    "-gencode", "arch=compute_100a,code=sm_100a",
                    f"-I{REPO / 'ppy_b200' / 'csrc'}", f"-I{REPO / 'include'}", "-o",
                    str(binary), str(source)], check=True, capture_output=True)
    widths = [int(w) for w in subprocess.run([str(binary)], check=True, capture_output=True,
                                             text=True).stdout.split()]
    assert widths == [w for _, w in CASES]
