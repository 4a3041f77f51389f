"""The standalone teaching trainer from Python: the same program as the fg_train executable (fg_train_main in
libflyguy_b200.so, csrc/fg_train.cu; the reference's flyguy_train, flyguy/native/flyguy_train.cu:631-788).

  python -m flyguy_b200.train NET.bin PARAMS.bin DATA_DIR OUT_PREFIX [--batch 512] [--lr 3e-4] ... [--steps N]
"""
from __future__ import annotations

import ctypes
import sys

from . import native


def main(argv: list[str] | None = None) -> int:
    args = ["fg_train"] + list(sys.argv[1:] if argv is None else argv)
    arr = (ctypes.c_char_p * len(args))(*[a.encode() for a in args])
    return int(native.lib().fg_train_main(len(args), arr))


if __name__ == "__main__":
    sys.exit(main())
