"""Prints the 32-entry table of the C library's expf algorithm (oracle/
esm_oracle_avx.c, esm-cpp_b200/csrc/refmath.cu): 2^(i/32) rounded to the
nearest double, as bits, minus i << 47 (the integer part of k/32 is added to
the exponent at run time).  Computed with 60-digit decimal arithmetic;
float(Decimal) rounds correctly.  TEST INFRASTRUCTURE and a build aid: the
table is written into both sources.

    python oracle/gen_exp2_table.py
"""
import struct
from decimal import Decimal, getcontext


def table():
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    out = []
    for i in range(32):
        f = float((ln2 * Decimal(i) / Decimal(32)).exp())
        bits = struct.unpack("<Q", struct.pack("<d", f))[0]
        out.append((bits - (i << 47)) & 0xFFFFFFFFFFFFFFFF)
    return out


if __name__ == "__main__":
    t = table()
    for i in range(0, 32, 4):
        print("    " + ", ".join("0x%016xull" % x for x in t[i:i + 4]) + ",")
