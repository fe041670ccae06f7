"""The torch restatement of the reference's CPU path (oracle/cpu_torch.py), which bench.py times
as the CPU baseline, against the reference-generated fixtures: the compressor's bytes, indices
and fp16 values bit for bit, and the CPU forward against the reference's own forward outputs."""
import numpy as np
import pytest
import torch

from golden_io import case_names, load
from oracle import cpu_torch

CASES = case_names()


def _W(g):
    W = torch.from_numpy(g["W"])
    return W.to(torch.bfloat16) if g["dtype"] == "bf16" else W


@pytest.mark.parametrize("name", CASES)
def test_port_compressor_matches_reference_bytes(name):
    g = load(name)
    dp, sp = cpu_torch.compress_matrix(_W(g))
    assert tuple(dp["padded_shape"]) == g["padded_shape"]
    np.testing.assert_array_equal(dp["exponents"].numpy(), g["exponents"])
    np.testing.assert_array_equal(dp["signs"].numpy(), g["signs"])
    np.testing.assert_array_equal(dp["payload"].numpy(), g["payload"])
    assert sp["count"] == g["count"]
    np.testing.assert_array_equal(sp["block_idx"].numpy(), g["block_idx"])
    np.testing.assert_array_equal(sp["offset"].numpy(), g["offset"])
    np.testing.assert_array_equal(sp["value"].numpy().view(np.uint16), g["value_bits"])


@pytest.mark.parametrize("name", CASES)
def test_port_forward_matches_reference_outputs(name):
    g = load(name)
    dp = {"exponents": torch.from_numpy(g["exponents"]), "signs": torch.from_numpy(g["signs"]),
          "payload": torch.from_numpy(g["payload"]), "orig_shape": g["orig_shape"],
          "padded_shape": g["padded_shape"]}
    sp = {"block_idx": torch.from_numpy(g["block_idx"]), "offset": torch.from_numpy(g["offset"]),
          "value": torch.from_numpy(g["value"].copy()), "count": g["count"]}
    n, k = g["orig_shape"]
    rcv = cpu_torch.outlier_rcv(sp, g["padded_shape"], n, k)
    bias = torch.from_numpy(g["bias"]) if "bias" in g else None
    for X, xdt, Yref in g["xs"]:
        Xt = torch.from_numpy(X).to(torch.bfloat16 if xdt == "bf16" else torch.float32)
        Y = cpu_torch.fallback_forward(Xt, dp, rcv, bias)
        np.testing.assert_allclose(Y.float().numpy(), Yref, rtol=1e-2,
                                   atol=1e-2 * float(np.abs(Yref).max()) + 1e-6)
