"""Prints the double-double constants of ddmath.h: ln 2 as the sum of three doubles and
1/n! (n = 0..11) as (hi, lo) pairs, computed exactly with Python's decimal/fractions."""
import math
from decimal import Decimal, getcontext
from fractions import Fraction

getcontext().prec = 80


def split(x: Fraction, parts: int):
    out = []
    for _ in range(parts):
        d = float(x)
        out.append(d)
        x -= Fraction(d)
    return out


if __name__ == "__main__":
    ln2 = Fraction(Decimal(2).ln())
    print("VX_LN2_1..3:", *(v.hex() for v in split(ln2, 3)))
    print("VX_LOG2E:", float(1 / ln2).hex())
    for n in range(12):
        hi, lo = split(Fraction(1, math.factorial(n)), 2)
        print(f"1/{n}!:", hi.hex(), lo.hex())
