"""Drop-in module paths of the reference package (``kvserve_v1``).

Code and configurations written for KVServe name its module paths, most
importantly the connector's
``kv_connector_module_path="kvserve_v1.connector.compressed_kv_connector"``.
The directory returned by :func:`path` holds a ``kvserve_v1`` package whose
modules forward to this package's implementations, so that such
configurations run unchanged with this framework:

    PYTHONPATH=$(python -c "import kvserve_hpdps_b200.compat as c; print(c.path())")

It is not on the import path by default, so it never shadows a real
``kvserve_v1`` installation (the benchmark's reference arm imports one).
vLLM imports the connector module in its worker processes, which inherit
``PYTHONPATH``.
"""

import os


def path() -> str:
    """Directory to put on ``sys.path`` / ``PYTHONPATH``."""
    return os.path.dirname(os.path.abspath(__file__))
