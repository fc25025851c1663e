"""Prints the 2^(i/32) table of q3_expf.h from the mathematics.

Each entry is 2^(i/32) rounded to the nearest binary64 (Python's Decimal at 80
digits, then float(), which rounds correctly), with (i << 47) subtracted from
its bit pattern so that adding k << 47 for k = 32*e + i yields 2^(k/32).
tests/test_expf.py checks that q3_expf.h holds exactly these values.
"""
import struct
from decimal import Decimal, getcontext


def table():
    getcontext().prec = 80
    ln2 = Decimal(2).ln()
    out = []
    for i in range(32):
        d = float((ln2 * Decimal(i) / Decimal(32)).exp())
        u = struct.unpack("<Q", struct.pack("<d", d))[0]
        out.append((u - ((i << 52) // 32)) & 0xFFFFFFFFFFFFFFFF)
    return out


if __name__ == "__main__":
    print(", ".join("0x%016xULL" % t for t in table()))
