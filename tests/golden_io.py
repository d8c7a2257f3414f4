"""Load the committed golden vectors (produced by tests/golden/make_golden.py)."""
import glob
import json
import os

import numpy as np

from oracle.inputs import MoECase

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_python_dir() -> str | None:
    """The reference checkout's ``python/`` directory (the one holding the ``vesper``
    package), or None when it is not available: ``$VESPER_REFERENCE_PYTHON`` if set, else
    ``reference/python`` in the directory that holds this repository.  Only fixture
    generation and CPU tests that execute the reference use it; GPU tests never do."""
    d = os.environ.get("VESPER_REFERENCE_PYTHON") or os.path.join(
        os.path.dirname(REPO), "reference", "python")
    return d if os.path.isfile(os.path.join(d, "vesper", "model.py")) else None


def golden_names():
    """The MoE-layer goldens (dense FeedForward ones start with 'ffn_', pre-norm blocks 'ln_')."""
    return sorted(n for n in (os.path.basename(p)[:-4]
                              for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
                  if not n.startswith(("ffn_", "ln_", "bw_")))


def ffn_golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "ffn_*.npz")))


def bw_golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "bw_*.npz")))


def ln_golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "ln_*.npz")))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    case = MoECase(**json.loads(str(z["case"])))
    return case, {k: z[k] for k in z.files if k not in ("case", "torch_version")}
