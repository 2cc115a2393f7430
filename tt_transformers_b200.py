"""Import name for the package whose sources live in the folder `tt-transformers_b200/`.

A hyphen cannot appear in a Python module name, so this module loads that folder's
`__init__.py` under the name `tt_transformers_b200` and puts it in `sys.modules` in
its own place: `import tt_transformers_b200.engine` then finds
`tt-transformers_b200/engine/`.
"""

import importlib.util
import os
import sys

_folder = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tt-transformers_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_folder, "__init__.py"), submodule_search_locations=[_folder]
)
_package = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _package
_spec.loader.exec_module(_package)
