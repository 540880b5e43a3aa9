"""Import name for the package kept in ``elastic-sparse-attention_b200/``.

A directory name with hyphens cannot be imported directly, so this module
loads that directory as the package ``elastic_sparse_attention_b200`` and
replaces itself with it in ``sys.modules``:

    from elastic_sparse_attention_b200 import ElasticSparseAttention
"""
import importlib.util
import os
import sys

_PKG_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "elastic-sparse-attention_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR])
_module = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
