"""Tensor-parallel shards on one GPU: every rank's shard of every 12B-class linear at TP 2 and 8
runs through the kernels (no device-side wait gives up) and matches a PyTorch fp32
dequantize-then-matmul, and a shard compressed alone equals the slice of the whole compression."""
import pytest
import torch

from flashbfp_b200 import OABFCompressor, packed, tp, workloads
from flashbfp_b200.linear import check_device_errors, packed_linear

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    from flashbfp_b200 import build
    build.build()
    torch.backends.cuda.matmul.allow_tf32 = False


def _full(dp, sp):
    """fp32 W_full of the shard (dequantised blocks + outliers; pinned bit-exact elsewhere)."""
    from flashbfp_b200 import _lib
    L = _lib.lib()
    n, k = dp["orig_shape"]
    kpad, _ = dp["padded_shape"]
    dev = dp["exponents"].device
    W = torch.empty(n, k, dtype=torch.float32, device=dev)
    st = _lib.stream_ptr(dev)
    _lib.check(L.fbfp_dequant(_lib.ptr(dp["exponents"]), _lib.ptr(dp["signs"]), _lib.ptr(dp["payload"]),
                              n, k, kpad, _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "dequant")
    if sp["count"]:
        _lib.check(L.fbfp_scatter_outliers(_lib.ptr(sp["block_idx"]), _lib.ptr(sp["offset"]),
                                           _lib.ptr(sp["value"]), sp["count"], kpad, n, k,
                                           _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "scatter")
    return W


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (8, 7)])
@pytest.mark.parametrize("name", ["q_proj", "k_proj", "o_proj", "gate_proj", "down_proj"])
def test_shard_runs_and_matches(name, world, rank):
    n, k = workloads.GEMMA12B_LAYER[name]
    dev = torch.device("cuda", 0)
    comp = OABFCompressor()
    W = workloads.decode_weight(n, k, seed=n + k + rank, device=dev)
    dp, sp = tp.compress_shard(W, name, rank, world, comp)
    pw = packed.from_compressed(dp, sp, dev)
    k0, k1 = tp.input_range(name, k, rank, world)
    for m in (1, 16, 40):
        X = workloads.activations(m, k, seed=m, device=dev)[:, k0:k1]
        Y = packed_linear(X, pw)
        check_device_errors()
        ref = X.float() @ _full(dp, sp).t()
        rel = ((Y.float() - ref).norm() / ref.norm()).item()
        assert rel <= 5e-3, (name, world, rank, m, rel)


@pytest.mark.parametrize("name", ["v_proj", "up_proj", "o_proj"])
def test_shard_bytes_equal_slice_of_whole(name):
    n, k = workloads.GEMMA12B_LAYER[name]
    dev = torch.device("cuda", 0)
    comp = OABFCompressor()
    W = workloads.decode_weight(n, k, seed=5, device=dev)
    full = packed.from_compressed(*comp.compress_matrix_device(W), dev, build_tiles=False)
    for rank in range(4):
        dp, sp = tp.compress_shard(W, name, rank, 4, comp)
        sl = tp.slice_packed(full, name, rank, 4, tiles=False)
        assert torch.equal(dp["exponents"].reshape(-1), sl.exps)
        assert torch.equal(dp["signs"].reshape(-1), sl.signs)
        assert torch.equal(dp["payload"].reshape(-1, 2), sl.payload)
        assert torch.equal(sp["block_idx"].to(torch.int32), sl.coo[0])
        assert torch.equal(sp["offset"].to(torch.int32), sl.coo[1])
