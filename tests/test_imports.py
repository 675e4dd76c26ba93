"""Every module of the package imports on a machine without a GPU, and every
benchmark entry point parses its command line (catches import-time errors in
code whose GPU paths only run on a B200)."""
import importlib
import pkgutil
import sys

import pytest

import nexar_b200

MODULES = sorted(m.name for m in pkgutil.walk_packages(nexar_b200.__path__, "nexar_b200.")
                 if not m.name.split(".")[-1].startswith("_"))


@pytest.mark.parametrize("name", MODULES)
def test_module_imports(name):
    importlib.import_module(name)


@pytest.mark.parametrize("name", [m for m in MODULES if m.startswith("nexar_b200.bench.")])
def test_bench_help(name, monkeypatch, capsys):
    mod = importlib.import_module(name)
    monkeypatch.setattr(sys, "argv", [name, "--help"])
    with pytest.raises(SystemExit) as e:
        mod.main()
    assert e.value.code == 0
    assert "usage" in capsys.readouterr().out


def test_flagship_bench_help(monkeypatch, capsys):
    import bench
    monkeypatch.setattr(sys, "argv", ["bench.py", "--help"])
    with pytest.raises(SystemExit) as e:
        bench.parse()
    assert e.value.code == 0 and "--attention" in capsys.readouterr().out
