"""The constants of the GPU's expf (rabbit2_b200/csrc/exact_math.cuh), on CPU.

* The 2^(i/32) table: every entry recomputed with 60-digit decimal arithmetic,
  rounded to the nearest double, minus i << 47.
* The host probe: this process's libm expf is one of the two x86-64 glibc
  builds of the table method the GPU reproduces (the library reports which), and
  that build's value at the probe input is what the library expects.
(The GPU reproduction itself is checked against this libm on every float in
tests/test_exact_routing_gpu.py.)
"""
import ctypes as C
import os
import re
import struct
from decimal import Decimal, getcontext
from fractions import Fraction

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rabbit2_b200", "csrc",
                      "exact_math.cuh")


def header_table():
    text = open(HEADER).read()
    body = text[text.index("kExp2Tab32[32] = {"):]
    body = body[:body.index("};")]
    return [int(v, 16) for v in re.findall(r"0x([0-9a-f]{16})ull", body)]


def test_exp2_table_is_correctly_rounded():
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    want = []
    for i in range(32):
        v = float(Fraction((ln2 * i / 32).exp()))  # correctly rounded to double
        want.append(struct.unpack("<Q", struct.pack("<d", v))[0] - (i << 47))
    assert header_table() == want


def test_host_expf_is_one_of_the_two_builds():
    from rabbit2_b200 import moe
    libm = C.CDLL("libm.so.6")
    libm.expf.restype = C.c_float
    libm.expf.argtypes = [C.c_float]
    y = libm.expf(float.fromhex("-0x1.f8cbb2p+5"))
    fma, plain = float.fromhex("0x1.f45326p-92"), float.fromhex("0x1.f45324p-92")
    assert y in (fma, plain)
    assert moe.host_expf_variant() == (1 if y == fma else 0)
