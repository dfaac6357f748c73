"""mllm_b200.kernel_cases on a machine without a GPU: the command parses its cases and refuses to
run (no CPU stand-in for a kernel)."""
import pytest

torch = pytest.importorskip("torch")


def test_kernel_cases_refuses_without_a_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from mllm_b200 import kernel_cases
    for case in ("epilogue", "prefill", "decode", "ragged", "linear", "linear_fp8"):
        with pytest.raises(SystemExit, match="needs a CUDA device"):
            kernel_cases.main([case, "--iters", "1"])


def test_kernel_cases_rejects_unknown_cases():
    from mllm_b200 import kernel_cases
    with pytest.raises(SystemExit):
        kernel_cases.main(["no_such_kernel"])
