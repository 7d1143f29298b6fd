"""Shared fixtures.  `-m gpu` tests need a CUDA device (a B200); everything else runs on CPU."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "flashinfer-bench-moe_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)

# Output tolerance the build is held to (per element, allclose rule).
ATOL = 1e-2
RTOL = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def oracle_mod():
    subprocess.run(["make", "-s", "-C", ORACLE], check=True)
    import oracle as o
    return o


@pytest.fixture(scope="session")
def fbmoe_lib():
    subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)
    import fbmoe_lib as lib
    lib.load_library()
    return lib


@pytest.fixture(scope="session")
def workloads():
    import fbmoe_workloads as w
    return w


@pytest.fixture(scope="session")
def golden_weights_cpu(workloads):
    """The 32-expert weights the golden fixtures were generated with (seed 1000, CPU generator)."""
    return workloads.make_weights(32, 1000, "cpu")


def load_golden_moe(name):
    return np.load(os.path.join(GOLDEN, f"moe_{name}.npz"))


def golden_moe_names():
    return sorted(f[4:-4] for f in os.listdir(GOLDEN) if f.startswith("moe_") and f.endswith(".npz"))


def golden_routing_names():
    return sorted(f[8:-4] for f in os.listdir(GOLDEN) if f.startswith("routing_") and f.endswith(".npz"))


def rebuild_golden_inputs(workloads, name, weights_cache):
    """Regenerate a golden case's inputs on CPU and verify their checksums."""
    from make_golden import tensor_checksum
    z = load_golden_moe(name)
    wseed = int(z["weight_seed"])
    if wseed not in weights_cache:
        weights_cache[wseed] = workloads.make_weights(32, wseed, "cpu")
    inp = workloads.make_inputs(int(z["T"]), seed=int(z["seed"]), config=str(z["config"]), device="cpu",
                                E_local=32, local_expert_offset=int(z["offset"]),
                                routed_scaling_factor=float(z["scale"]), weights=weights_cache[wseed])
    for k, v in zip(z["checksum_keys"], z["checksum_vals"]):
        got = tensor_checksum(inp[str(k)])
        assert got == str(v), f"regenerated input {k} differs from the fixture's ({got} != {v})"
    ref = torch.from_numpy(z["out_bits"]).view(torch.bfloat16)
    return inp, ref, z


@pytest.fixture(scope="session")
def weights_cache():
    return {}
