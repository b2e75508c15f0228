"""Generate the constants of the correctly rounded expf shared by the device
(nightrun_b200/csrc/expf_cr.cuh) and the CPU oracle (oracle/expf_cr.h).

exp(x) = 2^(k/64) * exp(r),  k = round(x * 64/ln2),  r = x - k*ln2/64,
with 2^(j/64), j = 0..63, stored as double-double (hi + lo), computed here to
60 significant digits with Python's decimal module, and the reduction
constants split so that k*ln2/64 is removed with two FMAs. Prints C source.
"""
from decimal import Decimal, getcontext

getcontext().prec = 60
LN2 = Decimal(2).ln()


def dd(v):
    hi = float(v)
    lo = float(v - Decimal(hi))
    return hi, lo


def main():
    rows = []
    for j in range(64):
        v = (LN2 * j / 64).exp()
        rows.append(dd(v))
    ln2_64 = LN2 / 64
    hi, lo = dd(ln2_64)
    inv = float(64 / LN2)
    print(f"// 64/ln2, ln2/64 = LN2_64_HI + LN2_64_LO")
    print(f"#define EXPCR_INV_LN2_64 {inv.hex()}")
    print(f"#define EXPCR_LN2_64_HI {hi.hex()}")
    print(f"#define EXPCR_LN2_64_LO {lo.hex()}")
    for n in (2, 3, 4, 5, 6):
        f = 1
        for i in range(2, n + 1):
            f *= i
        print(f"#define EXPCR_C{n} {float(Decimal(1) / f).hex()}")
    print("// 2^(j/64) = EXPCR_T[2j] + EXPCR_T[2j+1]")
    print("#define EXPCR_TABLE \\")
    for j, (h, l) in enumerate(rows):
        end = "" if j == 63 else " \\"
        print(f"  {h.hex()}, {l.hex()},{end}")


if __name__ == "__main__":
    main()
