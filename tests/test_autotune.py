"""Autotune decorator: the reference's tests (tests/test_autotune.py) plus validation cases."""

import pytest

from cutex_b200 import Config, autotune
from cutex_b200.autotune import read_autotune_spec


def test_autotune_decorator_records_validated_spec():
    @autotune(configs=[Config({"tile": 64}, name="tile64")], key=["m", "n"], warmup=2, rep=7)
    def kernel(m, n, tile=64):
        return m + n + tile

    spec = read_autotune_spec(kernel)
    assert spec is not None
    assert spec.key == ("m", "n")
    assert spec.configs[0].kwargs == {"tile": 64}
    assert spec.warmup == 2
    assert spec.rep == 7


def test_autotune_rejects_empty_search_space():
    with pytest.raises(ValueError, match="at least one"):
        autotune(configs=[], key=["m"])


@pytest.mark.parametrize("kwargs,match", [({"key": ["m", "m"]}, "unique"), ({"key": [""]}, "blank"),
                                          ({"key": ["m"], "warmup": -1}, "warmup"), ({"key": ["m"], "rep": 0}, "rep")])
def test_autotune_rejects_bad_specs(kwargs, match):
    with pytest.raises(ValueError, match=match):
        autotune(configs=[Config({"a": 1})], **kwargs)


def test_config_label_and_blank_name():
    assert Config({"tile_n": 256}).label == "{'tile_n': 256}"
    assert Config({"tile_n": 256}, name="n256").label == "n256"
    with pytest.raises(ValueError):
        Config({}, name="  ")


def test_gemm_search_space_is_attached_to_the_launcher():
    from cutex_b200.kernels.dense_gemm import GEMM_CONFIGS, mxfp8_gemm_launch

    spec = read_autotune_spec(mxfp8_gemm_launch)
    assert spec.key == ("m", "n", "k", "target")
    assert len(spec.configs) == len(GEMM_CONFIGS) >= 10
    assert len({c.name for c in spec.configs}) == len(spec.configs)
