"""Console plus rotating-file logging (reference: core/logging_config.py:36)."""

import logging
import logging.handlers
import os

_configured = False


def setup_logging(level=logging.INFO, log_dir=None, max_bytes=5 * 2 ** 20, backups=3):
    global _configured
    if _configured:
        return logging.getLogger()
    root = logging.getLogger()
    root.setLevel(level)
    fmt = logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s")
    ch = logging.StreamHandler()
    ch.setFormatter(fmt)
    root.addHandler(ch)
    if log_dir:
        os.makedirs(log_dir, exist_ok=True)
        fh = logging.handlers.RotatingFileHandler(os.path.join(log_dir, "b200serve.log"),
                                                  maxBytes=max_bytes, backupCount=backups)
        fh.setFormatter(fmt)
        root.addHandler(fh)
    _configured = True
    return root
