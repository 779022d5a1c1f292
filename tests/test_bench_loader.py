"""bench.py's step-input loader layout, on the CPU: the packed buffer holds every input at an
aligned offset without overlap, and the ranks' host-copy ranges tile it exactly (each rank
copies its range from host memory and pulls the others from its peers, so a gap or an
overlap would leave bytes unwritten or written twice)."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("total", [0, 1, 255, 256, 257, 4096 * 3 + 17, 807_075_840])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_rank_ranges_tile_the_buffer(total, world):
    b = bench.byte_parts(total, world)
    assert len(b) == world + 1 and b[0] == 0 and b[-1] == total
    assert all(b[i] <= b[i + 1] for i in range(world))
    assert all(x % 256 == 0 or x == total for x in b[:-1])  # a range clipped at the end is empty
    if total >= 256 * world:
        # balanced to within one alignment unit of 1/N
        sizes = [b[i + 1] - b[i] for i in range(world)]
        assert max(sizes) - min(sizes) <= 2 * 256


def test_packed_layout_keeps_inputs_aligned_and_disjoint():
    ins = [torch.zeros(128, 1536, 8, dtype=torch.bfloat16), torch.zeros(128, 1536, dtype=torch.int32),
           torch.zeros(128, 1536, dtype=torch.bool), torch.zeros(77, dtype=torch.float32)]
    offs, total = bench.pack_layout(ins)
    assert total % 256 == 0 and all(o % 256 == 0 for o in offs)
    spans = sorted((o, o + x.nbytes) for o, x in zip(offs, ins))
    assert all(spans[i][1] <= spans[i + 1][0] for i in range(len(spans) - 1))
    assert spans[-1][1] <= total
    # every input reads back through a typed view of the packed bytes
    buf = torch.arange(total, dtype=torch.int64).remainder(251).to(torch.uint8)
    for x, o in zip(ins, offs):
        v = buf[o:o + x.nbytes].view(x.dtype).view(x.shape)
        assert v.shape == x.shape and v.dtype == x.dtype
