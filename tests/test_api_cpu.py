"""API behaviour that needs no GPU: input validation and config errors (the reference's
tests/test_input_validation.py cases), generator seeding and RNG hygiene
(tests/test_side_effects.py), pruning and block sizing."""
import random

import pytest
import torch

from sumac_b200 import SumacConfig, SumacMethod, sumac_factorize
from sumac_b200.data import prune_zero_rows_cols, restore_zero_rows_cols


def valid_inputs():
    return {"S_index": torch.tensor([[0, 1], [0, 1]], dtype=torch.int64),
            "S_value": torch.tensor([1.0, 2.0]), "shape": (2, 2),
            "config": SumacConfig(verbose=False)}


@pytest.mark.parametrize(("replacement", "exception", "match"), [
    ({"S_index": torch.tensor([0, 1])}, ValueError, "shape"),
    ({"S_index": torch.tensor([[0, 1], [0, 1]], dtype=torch.float32)}, TypeError, "index dtype"),
    ({"S_value": torch.tensor([[1.0, 2.0]])}, ValueError, "S_value must have shape"),
    ({"S_value": torch.tensor([1.0])}, ValueError, "nnz dimensions"),
    ({"S_value": torch.tensor([1.0, float("inf")])}, ValueError, "finite"),
    ({"S_value": torch.tensor([1.0, -2.0])}, ValueError, "nonnegative"),
    ({"S_value": torch.tensor([1.0, 0.0])}, ValueError, "nonzero COO"),
    ({"shape": (2, 0)}, ValueError, "positive integers"),
    ({"S_index": torch.tensor([[0, 2], [0, 1]])}, ValueError, "row indices"),
    ({"S_index": torch.tensor([[0, 1], [0, 5]])}, ValueError, "column indices"),
    ({"S_index": torch.tensor([[0, 0], [0, 0]])}, ValueError, "duplicate"),
])
def test_invalid_sparse_inputs(replacement, exception, match):
    args = valid_inputs()
    args.update(replacement)
    with pytest.raises(exception, match=match):
        sumac_factorize(**args)


@pytest.mark.parametrize(("field", "value", "match"), [
    ("rank", 0, "rank"), ("max_iterations", -1, "max_iterations"), ("num_blocks", 0, "num_blocks"),
    ("cache_mb", float("nan"), "cache_mb"), ("dtype", torch.float16, "dtype"),
    ("eval_interval", 0, "eval_interval"), ("batch_blocks", 0, "batch_blocks"),
    ("learning_rate", -0.1, "learning_rate"), ("momentum", 1.0, "momentum"),
    ("tf32_mode", "fp16", "tf32_mode"),
])
def test_invalid_config_fields(field, value, match):
    with pytest.raises((TypeError, ValueError), match=match):
        SumacConfig(**{field: value}, verbose=False)


def test_float64_and_tf32_are_mutually_exclusive():
    with pytest.raises(ValueError, match="mutually exclusive"):
        SumacConfig(dtype=torch.float64, allow_tf32=True, verbose=False)


def test_initial_factors_must_be_provided_together():
    args = valid_inputs()
    args["A_init"] = torch.ones(2, args["config"].rank)
    with pytest.raises(ValueError, match="both be provided"):
        sumac_factorize(**args)


def test_initial_factor_shapes_are_validated():
    args = valid_inputs()
    args["A_init"] = torch.ones(1, args["config"].rank)
    args["B_init"] = torch.ones(2, args["config"].rank)
    with pytest.raises(ValueError, match="A_init must have shape"):
        sumac_factorize(**args)


def test_num_blocks_is_limited_by_effective_shape():
    args = valid_inputs()
    args["S_index"] = torch.tensor([[0], [0]])
    args["S_value"] = torch.tensor([1.0])
    args["config"].num_blocks = 2
    with pytest.raises(ValueError, match="effective shape"):
        sumac_factorize(**args)


def test_defaults_match_reference():
    c = SumacConfig(verbose=False)
    assert (c.method, c.rank, c.max_iterations, c.momentum, c.learning_rate, c.eval_interval) == \
        (SumacMethod.SALSA, 16, 25, 0.7, 0.1, 10)
    g = SumacConfig(method=SumacMethod.GD, verbose=False)
    assert g.eval_interval == 100


def test_config_does_not_touch_python_rng():
    state = random.getstate()
    SumacConfig(seed=42, verbose=False)
    assert random.getstate() == state


@pytest.mark.parametrize("seed", [42, None])
def test_get_generator_seeds_and_torch_rng(seed):
    torch.manual_seed(1729)
    before = torch.random.get_rng_state().clone()
    cfg = SumacConfig(method=SumacMethod.SALSA, seed=seed, device=torch.device("cpu"), verbose=False)
    gens = cfg.get_generator()
    torch.testing.assert_close(torch.random.get_rng_state(), before)
    seeds = tuple(g.initial_seed() for g in gens)
    if seed is None:
        assert len(set(seeds)) == 3
    else:
        assert seeds == (seed, seed + 1, seed + 2)


def test_gd_aux_generator_on_cpu():
    cfg = SumacConfig(method=SumacMethod.GD, seed=1, device=torch.device("cpu"), verbose=False)
    assert cfg.get_generator()[2].device.type == "cpu"


def test_block_sizes_from_cache_budget():
    cfg = SumacConfig(verbose=False, cache_mb=1)
    cfg.set_block_sizes(1000, 5000)
    assert cfg.num_blocks == 20 and cfg.cols_per_block == 250


def test_prune_and_restore_roundtrip():
    idx = torch.tensor([[0, 2, 2], [1, 1, 3]])
    new, rmask, cmask, m, n = prune_zero_rows_cols(idx, (4, 5))
    assert (m, n) == (2, 2)
    assert new.tolist() == [[0, 1, 1], [0, 0, 1]]
    A, B = torch.ones(2, 3), 2 * torch.ones(2, 3)
    Ao, Bo = restore_zero_rows_cols(A, B, 4, 5, 3, rmask, cmask)
    assert Ao[:, 0].tolist() == [1, 0, 1, 0] and Bo[:, 0].tolist() == [0, 2, 0, 2, 0]


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_cpu_fallback():
    args = valid_inputs()
    with pytest.raises(RuntimeError, match="no CPU implementation"):
        sumac_factorize(**args)


def test_init_salsa_factors_matches_reference_on_cpu(golden):
    """init_salsa_factors (training/salsa.py:36-78) run on the CPU with the seed-0 generator, on
    C1's data: the same draws and steps as the reference give its initial factors exactly
    (tests/golden/c1_gd.npz holds the reference's A0/B0)."""
    import numpy as np
    import torch

    from bench import make_c1
    from sumac_b200.salsa import init_salsa_factors
    g = golden("c1_gd")
    idx, vals, (m, n) = make_c1()
    gen = torch.Generator(device="cpu").manual_seed(0)
    A0, B0 = init_salsa_factors(torch.from_numpy(idx), torch.from_numpy(vals), m, n,
                                int(g["rank"]), gen)
    np.testing.assert_allclose(A0.numpy(), g["A0"], rtol=1e-5, atol=1e-6 * np.abs(g["A0"]).max())
    np.testing.assert_allclose(B0.numpy(), g["B0"], rtol=1e-5, atol=1e-6 * np.abs(g["B0"]).max())
