"""Native host runtime (``_mxrt``): checkpoint IO and the data pipeline.

``rt()`` imports the in-tree build, compiling it on first use when it is missing (it is plain
C++, so this works on machines without a GPU too).
"""

from __future__ import annotations

import importlib.util
import os
import threading

from .build import BUILD_DIR, EXT_NAME

_RT = None
_LOCK = threading.Lock()


def rt():
    global _RT
    if _RT is None:
        with _LOCK:
            if _RT is None:
                path = os.path.join(BUILD_DIR, EXT_NAME + ".so")
                if not os.path.exists(path):
                    from .build import build

                    build()
                spec = importlib.util.spec_from_file_location(EXT_NAME, path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                _RT = mod
    return _RT
