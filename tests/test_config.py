"""GICC_* environment parsing (native gicc::Config) and the rank-prefixed loggers."""
import logging
import subprocess
import sys

import pytest

from opengda_b200.utils.config import config, get_logger


def test_defaults(monkeypatch):
    for k in ("GICC_TIMEOUT_MS", "GICC_BOOTSTRAP_TIMEOUT_MS", "GICC_LOG_LEVEL", "GICC_CHECKS", "GICC_DISABLE_NVLS",
              "GICC_DEBUG", "GICC_SIGNAL_HEAP_BYTES"):
        monkeypatch.delenv(k, raising=False)
    c = config()
    assert c["timeout_ms"] == 5000 and c["bootstrap_timeout_ms"] == 0 and c["log_level"] == 1
    assert not c["checks"] and not c["disable_nvls"] and not c["debug_puts"] and c["signal_heap_bytes"] == 0


def test_values_are_parsed(monkeypatch):
    monkeypatch.setenv("GICC_TIMEOUT_MS", "1500")
    monkeypatch.setenv("GICC_BOOTSTRAP_TIMEOUT_MS", "0x2710")
    monkeypatch.setenv("GICC_LOG_LEVEL", "debug")
    monkeypatch.setenv("GICC_CHECKS", "1")
    monkeypatch.setenv("GICC_DISABLE_NVLS", "")  # present and empty = on
    monkeypatch.setenv("GICC_DEBUG", "off")
    monkeypatch.setenv("GICC_SIGNAL_HEAP_BYTES", str(8 << 20))
    c = config()
    assert c["timeout_ms"] == 1500 and c["bootstrap_timeout_ms"] == 10000 and c["log_level"] == 3
    assert c["checks"] and c["disable_nvls"] and not c["debug_puts"] and c["signal_heap_bytes"] == 8 << 20


@pytest.mark.parametrize("var,val", [("GICC_TIMEOUT_MS", "0"), ("GICC_TIMEOUT_MS", "-5"), ("GICC_TIMEOUT_MS", "5s"),
                                     ("GICC_BOOTSTRAP_TIMEOUT_MS", "10"), ("GICC_LOG_LEVEL", "loud"),
                                     ("GICC_CHECKS", "maybe"), ("GICC_SIGNAL_HEAP_BYTES", "100")])
def test_bad_values_name_the_variable(monkeypatch, var, val):
    monkeypatch.setenv(var, val)
    with pytest.raises(ValueError, match=var):
        config()


def test_native_log_is_rank_prefixed_and_filtered():
    code = ("from opengda_b200 import native; n = native(); "
            "n.log(2, 'hidden at warn'); n.log(0, 'shown error')")
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       env={**__import__("os").environ, "GICC_LOG_LEVEL": "warn"})
    assert p.returncode == 0, p.stderr
    assert "shown error" in p.stderr and "hidden at warn" not in p.stderr
    assert "[gicc error] shown error" in p.stderr


def test_python_logger(monkeypatch, capsys):
    monkeypatch.setenv("GICC_LOG_LEVEL", "info")
    monkeypatch.setenv("RANK", "3")
    lg = get_logger("test")
    assert lg.level == logging.INFO
    lg.info("hello")
    lg.debug("not shown")
    err = capsys.readouterr().err
    assert "[gicc r3 info] gicc.test: hello" in err and "not shown" not in err
