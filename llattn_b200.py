"""Import name of the package directory ``local-latent-attention_b200/``.

That directory name is not a Python identifier, so this module loads it under
the name ``llattn_b200`` (``import llattn_b200``; ``from llattn_b200 import
LocalLatentAttentionB200``) and replaces itself in ``sys.modules``.
"""

import importlib.util
import os
import sys

_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "local-latent-attention_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_DIR, "__init__.py"), submodule_search_locations=[_DIR]
)
_pkg = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _pkg
_spec.loader.exec_module(_pkg)
