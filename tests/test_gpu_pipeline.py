"""The whole product path on the B200, as the reference's suite drives a kernel file
(tests/pytorchsim-compile <k> --to verify): lower the Triton source into a kernel object, materialise the
spec's inputs as .raw files, run the object on the CUDA device (device registry "cuda"), and verify the
written .raw files against the spec's own torch reference (its rtol/atol).  Kernel files: tests/kernels/."""
import os
import tempfile

import pytest

from pytorchsim_triton_compiler.contract.kernel_spec import load_spec
from pytorchsim_triton_compiler.driver import compiler

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("kernel", ["relayout_scale.py", "row_softmax.py"])
def test_kernel_file_lowers_runs_and_verifies(kernel):
    spec = load_spec(os.path.join(HERE, "kernels", kernel))
    with tempfile.TemporaryDirectory() as wd:
        assert compiler.run(spec, wd) is True
