"""The GEMM kernel's barrier protocol under randomised schedules, on the CPU (tests/pipeline_model.py).

Every instantiated (cta_group, tile_n, stages, sf_buffers) combination, with
several tile counts and K-stage counts (ring wrap inside a tile and across
tiles, both TMEM accumulators and their overlap), must finish without a
deadlock or a data hazard under many random interleavings of the roles, the
TMA copies and the tensor pipe. Each planted mistake must be caught.
"""

import itertools

import pytest

from tests.pipeline_model import Mutation, ProtocolError, Shape, simulate

# (cta_group, tile_n, stages, sf_buffers) of the instantiated kernels (cutex_abi.cu, g_variants).
BUILDS = sorted({
    (2, 256, 6, 1), (2, 256, 5, 1), (2, 256, 6, 2), (2, 256, 4, 1), (2, 128, 6, 1), (2, 128, 8, 1),
    (1, 256, 4, 1), (1, 256, 3, 1), (1, 128, 6, 1), (1, 128, 5, 1), (1, 128, 4, 2), (1, 128, 5, 2),
    (1, 128, 6, 2), (1, 256, 3, 2), (1, 256, 4, 2), (2, 256, 4, 2), (2, 256, 5, 2), (2, 256, 6, 4),
    (2, 256, 5, 4),
})


@pytest.mark.parametrize("build", BUILDS, ids=lambda b: "cg{}_n{}_s{}_f{}".format(*b))
def test_protocol_has_no_hazard_or_deadlock(build):
    cg, tile_n, stages, sf = build
    for tiles, k_blocks in itertools.product((1, 2, 3, 5), (1, 2, stages - 1, stages + 1, 2 * stages + 3)):
        if k_blocks < 1:
            continue
        shape = Shape(cg, tile_n, stages, sf, tiles, k_blocks)
        for seed in range(10):
            simulate(shape, seed)


def test_overlapping_accumulators_are_exercised():
    # tile_n = 256 leaves no room for two disjoint accumulators: buffer 1 overlaps buffer 0.
    sh = Shape(2, 256, 6, 1, 3, 4)
    assert sh.overlap and sh.acc1_col == 240 and sh.first_chunk(0) == 3
    assert not Shape(1, 128, 6, 2, 3, 4).overlap


MUTATIONS = {
    "mma_waits_own_buffer": Shape(2, 256, 6, 1, 4, 3),
    "epilogue_skips_overlap_first": Shape(1, 256, 4, 1, 4, 3),
    "release_after_first_chunk_only": Shape(1, 128, 6, 1, 4, 3),
    "producer_parity_unflipped": Shape(1, 128, 4, 1, 2, 5),
    "commit_before_last_mma": Shape(1, 128, 2, 1, 3, 5),
}


@pytest.mark.parametrize("name", sorted(MUTATIONS))
def test_planted_mistakes_are_caught(name):
    shape = MUTATIONS[name]
    caught = 0
    for seed in range(200):
        try:
            simulate(shape, seed, Mutation(**{name: True}))
        except ProtocolError:
            caught += 1
    assert caught > 0, f"{name}: no schedule exposed the planted mistake"
