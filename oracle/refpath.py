"""Where the reference checkout is (test infrastructure: the golden-fixture generator and the build of the
reference's decode kernels read it; nothing on the GPU box does).

$QK_REFERENCE_DIR names the checkout's root (the folder holding qwen3-8b-fp8_rtx-5090/); without it, a folder
called `reference` beside this repository is used.
"""
import os

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE = "qwen3-8b-fp8_rtx-5090"


def reference_root() -> str:
    return os.environ.get("QK_REFERENCE_DIR") or os.path.join(os.path.dirname(REPO), "reference")


def engine_dir() -> str:
    """The reference engine's folder (model.py, generate.py, kernels/decode.cu)."""
    return os.path.join(reference_root(), ENGINE)
