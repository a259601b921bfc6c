"""Logging for kvserve_hpdps_b200.

``KVSERVE_LOG_LEVEL`` (ERROR | WARNING | INFO | DEBUG, default WARNING) sets
the verbosity, like the reference logger (kvserve_v1/utils/logger.py:20-21).
Messages go through the standard ``logging`` module under the
``kvserve_hpdps_b200`` logger so that vLLM's handlers pick them up.
"""

from __future__ import annotations

import logging
import os

_LEVELS = {"ERROR": logging.ERROR, "WARNING": logging.WARNING,
           "INFO": logging.INFO, "DEBUG": logging.DEBUG}

_root = logging.getLogger("kvserve_hpdps_b200")
_root.setLevel(_LEVELS.get(os.environ.get("KVSERVE_LOG_LEVEL", "WARNING").upper(),
                           logging.WARNING))
if not _root.handlers:
    _h = logging.StreamHandler()
    _h.setFormatter(logging.Formatter("[kvs %(levelname)s %(name)s] %(message)s"))
    _root.addHandler(_h)
    _root.propagate = False


def get_logger(name: str) -> logging.Logger:
    """Child logger under the package logger."""
    if not name.startswith("kvserve_hpdps_b200"):
        name = "kvserve_hpdps_b200." + name
    return logging.getLogger(name)


def set_log_level(level: str) -> None:
    _root.setLevel(_LEVELS.get(level.upper(), logging.WARNING))


_log = get_logger("kvs")


def log_debug(msg: str) -> None:
    _log.debug(msg)


def log_info(msg: str) -> None:
    _log.info(msg)


def log_warning(msg: str) -> None:
    _log.warning(msg)


def log_error(msg: str) -> None:
    _log.error(msg)
