"""Verbosity-gated logging helpers (role of kvserve_v1/utils/logger.py:10-57).

The level comes from ``KVSERVE_LOG_LEVEL`` (ERROR, WARNING, INFO, DEBUG;
default WARNING) and can be changed at run time with :func:`set_log_level`.
Messages go through the standard :mod:`logging` logger ``"kvserve_b200"``
so applications can route them like any other log record.
"""
from __future__ import annotations

import logging
import os
from enum import IntEnum


class LogLevel(IntEnum):
    ERROR = 0
    WARNING = 1
    INFO = 2
    DEBUG = 3


_TO_LOGGING = {LogLevel.ERROR: logging.ERROR, LogLevel.WARNING: logging.WARNING, LogLevel.INFO: logging.INFO,
               LogLevel.DEBUG: logging.DEBUG}

_logger = logging.getLogger("kvserve_b200")
if not _logger.handlers:
    _h = logging.StreamHandler()
    _h.setFormatter(logging.Formatter("[%(levelname)s] %(message)s"))
    _logger.addHandler(_h)
    _logger.propagate = False


def _level_from_env() -> LogLevel:
    name = os.environ.get("KVSERVE_LOG_LEVEL", "WARNING").strip().upper()
    return LogLevel[name] if name in LogLevel.__members__ else LogLevel.WARNING


_level = _level_from_env()
_logger.setLevel(_TO_LOGGING[_level])


def set_log_level(level: LogLevel) -> None:
    global _level
    _level = LogLevel(level)
    _logger.setLevel(_TO_LOGGING[_level])


def get_log_level() -> LogLevel:
    return _level


def log_debug(message: str) -> None:
    _logger.debug(message)


def log_info(message: str) -> None:
    _logger.info(message)


def log_warning(message: str) -> None:
    _logger.warning(message)


def log_error(message: str) -> None:
    """Errors are always emitted, whatever the level."""
    if _logger.level > logging.ERROR:
        _logger.log(logging.CRITICAL, message)
    else:
        _logger.error(message)
