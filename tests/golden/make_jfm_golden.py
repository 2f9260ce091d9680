"""Copies the reference's frozen JFM v2 golden package (hex text, one file per
package file) into tests/golden/jfm-v2-golden/ so the loader tests run where
the reference tree is absent.

Source: runtime/engines/native/tests/fixtures/jfm-v2-golden/*.hex in the
reference (decoded by runtime/engines/native/tests/engine_test.cpp:95-115).
The hex is data (a byte contract), copied verbatim.
"""
import shutil
import sys
from pathlib import Path

if len(sys.argv) != 2:
    sys.exit("usage: make_jfm_golden.py <reference checkout>/runtime/engines/native/tests/fixtures/jfm-v2-golden")
SOURCE = Path(sys.argv[1])
TARGET = Path(__file__).resolve().parent / "jfm-v2-golden"

if __name__ == "__main__":
    TARGET.mkdir(exist_ok=True)
    for name in ["manifest.jfm", "metadata.gguf", "input.jfs", "layer-00000.jfs",
                 "layer-00001.jfs", "output.jfs"]:
        shutil.copyfile(SOURCE / f"{name}.hex", TARGET / f"{name}.hex")
    print("copied", len(list(TARGET.glob("*.hex"))), "files")
