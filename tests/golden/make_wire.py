"""Copies the reference helper's wire fixtures (Tests/Fixtures/wire/dictation*.txt in the
reference repository) into tests/golden/wire/, the bytes tests/test_worker_wire.py compares
against.  Run where the reference tree is available:

    python tests/golden/make_wire.py /path/to/reference
"""
import shutil
import sys
from pathlib import Path

NAMES = ("dictation.txt", "dictation-load-failed.txt")

if __name__ == "__main__":
    src = Path(sys.argv[1]) / "Tests" / "Fixtures" / "wire"
    dst = Path(__file__).resolve().parent / "wire"
    dst.mkdir(exist_ok=True)
    for name in NAMES:
        shutil.copyfile(src / name, dst / name)
        print("copied", name)
