"""log_info / log_warn through the "WeightFerry" logger (utils/logging.py of the reference)."""

import logging

_log = logging.getLogger("WeightFerry")


def log_info(msg):
    _log.info("[WeightFerry] %s", msg)


def log_warn(msg):
    _log.warning("[WeightFerry] %s", msg)
