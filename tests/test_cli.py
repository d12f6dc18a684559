"""CLI argument handling (CPU only): openquant/cli.py:6-92 surface."""
import pytest

from openquant.cli import main


def test_version(capsys):
    with pytest.raises(SystemExit) as e:
        main(["--version"])
    assert e.value.code == 0
    assert "OpenQuant 0.5.0" in capsys.readouterr().out


def test_help_without_command(capsys):
    assert main([]) == 0
    assert "usage" in capsys.readouterr().out


@pytest.mark.parametrize("argv", [["cpu", "--rows", "0"], ["cpu", "--cols", "-3"], ["nosuch"]])
def test_bad_arguments(argv):
    with pytest.raises(SystemExit) as e:
        main(argv)
    assert e.value.code == 2


def test_report_validation_before_gpu():
    from openquant.report import make_cpu_report

    for rows, cols, group in [(0, 8, 4), (3, 0, 4), (2, 3, 3)]:
        with pytest.raises(ValueError):
            make_cpu_report(rows, cols, group_size=group)
