"""The C++ host API (include/ultravec_b200.hpp), on the CPU: every method
against a stand-in of the C ABI that checks the library's argument
contract (tests/cpp/mock_uv.cpp), its host-side arithmetic against the
oracle, and the header linked against the real library on a machine
without a GPU."""
from __future__ import annotations

import pytest

import cppbuild


def test_cpp_api_against_the_c_abi_stand_in(tmp_path):
    exe = cppbuild.build(tmp_path, "test_hpp_mock", ["test_hpp_mock.cpp", "mock_uv.cpp"],
                         link_library=False)
    out = cppbuild.run(exe)
    assert out.startswith("ok ") and int(out.split()[1]) >= 90


def test_cpp_reconstruct_normalization_is_the_oracles(tmp_path, oracle):
    """reconstruct_unit's host arithmetic (l2_norm in the reference's order,
    the centroid recomposition) gives the oracle's bits on decoded records,
    built with FMA contraction allowed."""
    exe = cppbuild.build(tmp_path, "test_hpp_oracle", ["test_hpp_oracle.cpp"],
                         link_library=False, link_oracle=True,
                         extra_flags=["-O2", "-mfma", "-ffp-contract=fast"])
    out = cppbuild.run(exe)
    assert out.startswith("ok ") and int(out.split()[1]) == 240


def test_cpp_api_links_the_library_and_fails_cleanly_without_a_gpu(tmp_path, uv):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    exe = cppbuild.build(tmp_path, "test_hpp_nogpu", ["test_hpp_nogpu.cpp"], link_library=True)
    assert cppbuild.run(exe).strip() == "ok"
