import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def pool(oracle):
    # the reference's generic (scalar) Q8_0 order: the GPU path reproduces it bit for bit
    p = oracle.Pool(threads=min(8, os.cpu_count() or 1), kernel=oracle.KERNEL_SCALAR)
    yield p
    p.close()


@pytest.fixture(scope="session")
def pool_avx2(oracle):
    # the reference's AVX2 int8 routine (expert_kernel.rs:163-191): same integers, other f32 order
    p = oracle.Pool(threads=min(8, os.cpu_count() or 1), kernel=oracle.KERNEL_AVX2)
    yield p
    p.close()


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "golden_v1.json")) as f:
        return json.load(f)
