"""The C++ drop-in: ClusterLM's BackendAdapter / ExecutionDomain / Drafter served by the b200 backend.

tests/backend/backend_parity.cpp (built as oracle/_ref/backend_parity, linking the reference's own domain code and
clusterlm_b200/backend/b200_backend.cpp) runs the reference pipeline and the b200 pipeline over the same fixture
model and compares them: generation traces (logits within 1e-4 absolute, same argmax, same accepted counts and
tokens), mixed reference/b200 stage pipelines, admission/commit/abort rules and the GPU MTP drafter.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "oracle", "_ref", "backend_parity")
BACKEND_SO = os.path.join(ROOT, "clusterlm_b200", "lib", "libclm_b200_backend.so")


def _need_driver():
    if not os.path.exists(DRIVER):
        pytest.skip("backend_parity not built (needs the reference sources at build time)")


def _has_gpu():
    import torch

    return torch.cuda.is_available()


def test_backend_library_exports_the_factory():
    if not os.path.exists(BACKEND_SO):
        pytest.skip("libclm_b200_backend.so not built (needs the reference sources at build time)")
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", BACKEND_SO], capture_output=True, text=True).stdout
    assert "clusterlm::backends::make_b200_backend(" in out
    assert "clusterlm::backends::make_b200_mtp_drafter(" in out


def test_backend_reports_hardware_unavailable_without_gpu(tmp_path):
    _need_driver()
    if _has_gpu():
        pytest.skip("a GPU is present")
    r = subprocess.run([DRIVER, str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode != 0
    assert "FAIL backend info" in r.stdout  # hardware_available is false
    assert "HARDWARE_UNAVAILABLE" in r.stdout  # create_domain refuses with kHardwareUnavailable


@pytest.mark.gpu
def test_dropin_pipelines_match_reference(tmp_path):
    _need_driver()
    r = subprocess.run([DRIVER, str(tmp_path), "--bench"], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("quant", ["q4_k", "q8_0"])
def test_llama_manifest_pipeline_through_execution_domain(tmp_path, oracle, quant):
    """The Llama family behind ExecutionDomain: a llama GGUF file (written by gguf-py in llama.cpp's tensor names) is
    turned into a ModelManifest by the reference's own build_llama_manifest; a prefix / middle / tail pipeline of b200
    domains binds its tensors from an ObjectResolver over the file and must give the logits of a whole-model engine
    loaded from the same file, bit for bit; the domains' requirements and the MTP proposal are checked too."""
    import sys

    _need_driver()
    pytest.importorskip("gguf")
    sys.path.insert(0, os.path.dirname(__file__))
    from test_gguf_gpu import _write_model
    from test_llama_gpu import small_geo

    geo = small_geo(quant, n_layers=4)
    path = tmp_path / "llama.gguf"
    _write_model(path, oracle, geo)
    r = subprocess.run([DRIVER, str(tmp_path), "--llama", str(path)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout
