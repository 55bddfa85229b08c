"""The robotcpp::Model adapter (robot.cpp_b200/adapter), compiled against the reference's own
src/models/model.h. Its C++ test program checks the observation -> engine input conversion and error paths
on CPU, and on a B200 that Model::predict() equals b2s_bitvla_predict of the same inputs bit for bit.

The program is built by __graft_entry__.build() where the reference's header is available (the include path
is the adapter Makefile's ROBOTCPP_SRC); the built binary travels with the tree.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "robot.cpp_b200", "adapter", "bitvla_model_test")

needs_bin = pytest.mark.skipif(not os.path.exists(BIN),
                               reason="adapter test program not built (needs the reference's models/model.h)")


def run(mode):
    p = subprocess.run([BIN, mode], capture_output=True, text=True, timeout=600)
    return p.returncode, p.stdout + p.stderr


@needs_bin
def test_adapter_input_conversion_cpu(b2s):
    rc, out = run("--cpu")
    assert rc == 0 and out.strip().endswith("OK"), out


@needs_bin
@pytest.mark.gpu
def test_adapter_predict_matches_library(b2s):
    rc, out = run("--gpu")
    assert rc == 0 and out.strip().endswith("OK"), out
