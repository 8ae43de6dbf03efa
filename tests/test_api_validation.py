"""Frontend validation (tonari src/tonari/api.py:176-196 and
src/tonari/_torch_frontend.py:25-75): same exception types and messages,
raised before any device work."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tonari_b200 import neighbor_list

ARGS = (torch.zeros((1, 3)), torch.zeros((3, 3)), torch.zeros(3, dtype=torch.bool), 1.0)


def test_quantities_and_algorithm_validation():
    with pytest.raises(TypeError, match="quantities must be a string"):
        neighbor_list(None, *ARGS)
    with pytest.raises(ValueError, match="unsupported quantities: 'x'"):
        neighbor_list("ix", *ARGS)
    with pytest.raises(TypeError, match="algorithm must be a string"):
        neighbor_list("PS", *ARGS, algorithm=1)
    with pytest.raises(ValueError, match="algorithm must be"):
        neighbor_list("PS", *ARGS, algorithm="octree")


@pytest.mark.parametrize("value,error", [(True, TypeError), (1.5, TypeError), (0, ValueError)])
def test_cpu_threads_validation(value, error):
    with pytest.raises(error):
        neighbor_list("PS", *ARGS, cpu_threads=value)


@pytest.mark.parametrize("option", ["sorted", "half_list", "include_self"])
def test_boolean_options_require_bool(option):
    with pytest.raises(TypeError, match="sorted, half_list, and include_self must be bool"):
        neighbor_list("PS", *ARGS, **{option: 1})


def test_shape_dtype_and_cutoff_validation():
    with pytest.raises(ValueError, match="positions must have shape"):
        neighbor_list("PS", torch.zeros((2, 2)), *ARGS[1:])
    with pytest.raises(ValueError, match="single-structure cell"):
        neighbor_list("PS", ARGS[0], torch.zeros((2, 3)), *ARGS[2:])
    with pytest.raises(ValueError, match="dtype float32 or float64"):
        neighbor_list("PS", torch.zeros((1, 3), dtype=torch.int32), *ARGS[1:])
    with pytest.raises(ValueError, match="cutoff must be finite and positive"):
        neighbor_list("PS", *ARGS[:3], float("inf"))
    with pytest.raises(ValueError, match="same dtype"):
        neighbor_list("PS", ARGS[0], torch.zeros((3, 3), dtype=torch.float64), *ARGS[2:])
    with pytest.raises(TypeError, match="must all be PyTorch tensors"):
        neighbor_list("PS", ARGS[0], np.zeros((3, 3)), *ARGS[2:])


def test_cpu_inputs_are_not_served_by_the_cuda_provider():
    with pytest.raises(RuntimeError, match="CUDA provider only"):
        neighbor_list("PS", *ARGS)
    with pytest.raises(RuntimeError, match="CUDA provider only"):
        neighbor_list("PS", np.zeros((1, 3)), np.zeros((3, 3)), np.zeros(3, dtype=bool), 1.0)
    assert neighbor_list.__module__ == "tonari_b200.api"
