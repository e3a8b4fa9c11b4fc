"""Import of the Hy-Nomas reference itself, where a checkout is named by ``HY_NOMAS_REF``
(TEST INFRASTRUCTURE: used by the golden-fixture generator, the installer test and the
reference arm of ``bench.py``; never by the product package).

``hymm.models.dit.nomas_cpt`` imports ``diffusers`` only for two base classes and a decorator
(``ModelMixin``, ``ConfigMixin``, ``register_to_config``).  ``diffusers`` is not installed
here, so a stand-in package with those three names is put on ``sys.path`` ahead of the
reference; everything else the path needs imports unchanged.
"""
import os
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
_DONE = False


def checkout() -> Path | None:
    """The reference checkout named by HY_NOMAS_REF (the directory holding ``hymm/``), or None."""
    ref = os.environ.get("HY_NOMAS_REF")
    if ref and (Path(ref) / "hymm").is_dir():
        return Path(ref)
    return None


def install_stub() -> Path:
    """Make ``hymm`` importable: the ``diffusers`` stand-in, the checkout and this repository
    on ``sys.path``.  Raises ``RuntimeError`` when HY_NOMAS_REF names no checkout."""
    global _DONE
    ref = checkout()
    if ref is None:
        raise RuntimeError("set HY_NOMAS_REF to the Hy-Nomas reference checkout (the directory holding hymm/)")
    if not _DONE:
        stub = Path(tempfile.mkdtemp(prefix="hyb_stub_"))
        (stub / "diffusers" / "models").mkdir(parents=True)
        (stub / "diffusers" / "__init__.py").write_text("")
        (stub / "diffusers" / "models" / "__init__.py").write_text(
            "import torch.nn as nn\nclass ModelMixin(nn.Module):\n    pass\n")
        (stub / "diffusers" / "configuration_utils.py").write_text(
            "class ConfigMixin:\n    pass\ndef register_to_config(fn):\n    return fn\n")
        sys.path.insert(0, str(stub))
        sys.path.insert(0, str(ref))
        sys.path.insert(0, str(REPO))
        _DONE = True
    return ref
