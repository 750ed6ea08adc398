"""Configuration and logging for Python code of the framework.

``config()`` returns the runtime's parsed and range-checked ``GICC_*`` environment (the
same parser the native library runs at ``Runtime`` start; a bad value raises
``ValueError`` naming the variable).  ``get_logger(name)`` returns a logger whose records
carry the rank (``[gicc r3 info] name: ...``) and whose level follows ``GICC_LOG_LEVEL``
(error | warn | info | debug or 0..3; default warn).

Variables: GICC_TIMEOUT_MS (device wait bound), GICC_BOOTSTRAP_TIMEOUT_MS,
GICC_LOG_LEVEL, GICC_CHECKS (bounds-checked puts), GICC_DISABLE_NVLS, GICC_DEBUG (log host
transfers), GICC_SIGNAL_HEAP_BYTES; plus the bootstrap's GICC_RANK / GICC_SIZE /
GICC_LOCAL_RANK / GICC_LOCAL_SIZE / GICC_BOOTSTRAP_ADDR (or torchrun's RANK, WORLD_SIZE,
LOCAL_RANK, MASTER_ADDR / MASTER_PORT).
"""
from __future__ import annotations

import logging
import os
import sys

_LEVELS = {"error": logging.ERROR, "0": logging.ERROR, "warn": logging.WARNING, "warning": logging.WARNING,
           "1": logging.WARNING, "info": logging.INFO, "2": logging.INFO, "debug": logging.DEBUG,
           "3": logging.DEBUG}


def config() -> dict:
    from .. import native

    return dict(native().config())


def log_level() -> int:
    v = os.environ.get("GICC_LOG_LEVEL", "warn").strip().lower()
    if v not in _LEVELS:
        raise ValueError(f"GICC_LOG_LEVEL={v}: expected error|warn|info|debug|0..3")
    return _LEVELS[v]


def _rank() -> str:
    for k in ("GICC_RANK", "RANK"):
        if k in os.environ:
            return os.environ[k]
    return "?"


class _RankFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        lvl = {logging.ERROR: "error", logging.WARNING: "warn", logging.INFO: "info"}.get(record.levelno, "debug")
        return f"[gicc r{_rank()} {lvl}] {record.name}: {record.getMessage()}"


def get_logger(name: str) -> logging.Logger:
    lg = logging.getLogger(f"gicc.{name}")
    if not getattr(lg, "_gicc_configured", False):
        h = logging.StreamHandler(sys.stderr)
        h.setFormatter(_RankFormatter())
        lg.addHandler(h)
        lg.propagate = False
        lg._gicc_configured = True
    lg.setLevel(log_level())
    return lg
