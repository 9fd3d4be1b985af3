"""Generate dft_codelets.cuh: fully unrolled forward DFT butterflies for the
radices the B200 Stockham kernels use.

Each codelet ``dft<R>(v)`` computes, in place on ``v[0..R)``,
    y[k] = sum_n v[n] * exp(-2*pi*i*n*k/R).
Odd primes use the symmetric pair form y[k] = A_k - i B_k, y[R-k] = A_k + i B_k
with A_k = x0 + sum_n (x_n + x_{R-n}) cos(2 pi n k / R) and
B_k = sum_n (x_n - x_{R-n}) sin(2 pi n k / R).  Composite radices use one
Cooley-Tukey split R = R1 * R2 with literal twiddles; trivial twiddles
(+-1, +-i, (+-1 +-i)/sqrt2) are emitted without multiplications.
Inverse transforms are obtained by the caller through conjugation.

Constants are computed with Python decimal arithmetic at 60 digits and emitted as
``kc<T>(hi, lo)``: hi is the correctly rounded double of the constant and lo the
correctly rounded double of the remainder, both as exact hex-float literals.  f32 and
f64 codelets use hi; the double-double type takes both words (its 106-bit constants).

Usage: python gen_codelets.py  (writes dft_codelets.cuh beside this file)
"""
import os
from decimal import Decimal, getcontext

getcontext().prec = 60
HERE = os.path.dirname(os.path.abspath(__file__))
PI = Decimal("3.14159265358979323846264338327950288419716939937510582097494459")


def _sin_cos(a):
    """Taylor series of sin and cos at |a| <= 2 pi in 60-digit decimal arithmetic."""
    s, c = Decimal(0), Decimal(0)
    term = a
    k = 1
    while True:
        s += term
        term = -term * a * a / ((k + 1) * (k + 2))
        k += 2
        if abs(term) < Decimal(10) ** -58:
            break
    term = Decimal(1)
    k = 0
    while True:
        c += term
        term = -term * a * a / ((k + 1) * (k + 2))
        k += 2
        if abs(term) < Decimal(10) ** -58:
            break
    return s, c

PRIMES = [2, 3, 5, 7, 11, 13]
SPLITS = {4: (2, 2), 8: (2, 4), 9: (3, 3), 16: (4, 4), 6: (2, 3), 10: (2, 5), 12: (3, 4), 14: (2, 7),
          15: (3, 5), 32: (4, 8)}
RADICES = [2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 32]


def lit(x):
    x = x.quantize(Decimal(10) ** -45)  # drop the series' last-digit noise (exact values stay exact)
    hi = float(x)
    lo = float(x - Decimal(hi))
    return f"kc<T>({hi.hex()}, {lo.hex()})"


def cs(m, r):
    a = 2 * PI * Decimal(m % r) / Decimal(r)
    if a > PI:
        a -= 2 * PI
    s, c = _sin_cos(a)
    return c, s


def emit_prime(r):
    lines = [f"template <typename T> B200FFT_HD void dft{r}(cplx<T>* v) {{"]
    if r == 2:
        lines += [
            "    const cplx<T> a = v[0], b = v[1];",
            "    v[0].x = a.x + b.x; v[0].y = a.y + b.y;",
            "    v[1].x = a.x - b.x; v[1].y = a.y - b.y;",
            "}",
        ]
        return lines
    h = (r - 1) // 2
    lines.append("    const cplx<T> x0 = v[0];")
    for n in range(1, h + 1):
        lines.append(f"    const T s{n}x = v[{n}].x + v[{r - n}].x, s{n}y = v[{n}].y + v[{r - n}].y;")
        lines.append(f"    const T d{n}x = v[{n}].x - v[{r - n}].x, d{n}y = v[{n}].y - v[{r - n}].y;")
    sx = " + ".join(f"s{n}x" for n in range(1, h + 1))
    sy = " + ".join(f"s{n}y" for n in range(1, h + 1))
    lines.append(f"    v[0].x = x0.x + {sx}; v[0].y = x0.y + {sy};")
    for k in range(1, h + 1):
        ax, ay, bx, by = ["x0.x"], ["x0.y"], [], []
        for n in range(1, h + 1):
            c, s = cs(n * k, r)
            ax.append(f"{lit(c)} * s{n}x")
            ay.append(f"{lit(c)} * s{n}y")
            bx.append(f"{lit(s)} * d{n}x")
            by.append(f"{lit(s)} * d{n}y")
        lines.append(f"    {{ const T ax = {' + '.join(ax)}; const T ay = {' + '.join(ay)};")
        lines.append(f"      const T bx = {' + '.join(bx)}; const T by = {' + '.join(by)};")
        lines.append(f"      v[{k}].x = ax + by; v[{k}].y = ay - bx;")
        lines.append(f"      v[{r - k}].x = ax - by; v[{r - k}].y = ay + bx; }}")
    lines.append("}")
    return lines


def twiddle_stmt(dst, m, r):
    """dst *= exp(-2 pi i m / r), with the trivial cases special-cased."""
    m %= r
    if m == 0:
        return []
    # reduce to eighths when exact
    if (8 * m) % r == 0:
        e = (8 * m) // r  # angle = -e*pi/4
        sq = lit(Decimal(2).sqrt() / 2)
        if e == 2:  # -i
            return [f"{{ const T q = {dst}.x; {dst}.x = {dst}.y; {dst}.y = -q; }}"]
        if e == 4:  # -1
            return [f"{dst}.x = -{dst}.x; {dst}.y = -{dst}.y;"]
        if e == 6:  # +i
            return [f"{{ const T q = {dst}.x; {dst}.x = -{dst}.y; {dst}.y = q; }}"]
        if e == 1:  # (1 - i)/sqrt2
            return [f"{{ const T a = {dst}.x, b = {dst}.y; {dst}.x = {sq} * (a + b); {dst}.y = {sq} * (b - a); }}"]
        if e == 3:  # (-1 - i)/sqrt2
            return [f"{{ const T a = {dst}.x, b = {dst}.y; {dst}.x = {sq} * (b - a); {dst}.y = -{sq} * (a + b); }}"]
        if e == 5:  # (-1 + i)/sqrt2
            return [f"{{ const T a = {dst}.x, b = {dst}.y; {dst}.x = -{sq} * (a + b); {dst}.y = {sq} * (a - b); }}"]
        if e == 7:  # (1 + i)/sqrt2
            return [f"{{ const T a = {dst}.x, b = {dst}.y; {dst}.x = {sq} * (a - b); {dst}.y = {sq} * (a + b); }}"]
    c, s = cs(m, r)
    return [f"{{ const T a = {dst}.x, b = {dst}.y; {dst}.x = a * {lit(c)} + b * {lit(s)}; "
            f"{dst}.y = b * {lit(c)} - a * {lit(s)}; }}"]


def emit_split(r):
    r1, r2 = SPLITS[r]
    lines = [f"template <typename T> B200FFT_HD void dft{r}(cplx<T>* v) {{"]
    lines.append(f"    cplx<T> t[{r}];")
    for n1 in range(r1):
        lines.append(f"    {{ cplx<T> u[{r2}];")
        for n2 in range(r2):
            lines.append(f"      u[{n2}] = v[{n1 + r1 * n2}];")
        lines.append(f"      dft{r2}<T>(u);")
        for k2 in range(r2):
            lines += ["      " + s for s in twiddle_stmt(f"u[{k2}]", n1 * k2, r)]
            lines.append(f"      t[{n1 * r2 + k2}] = u[{k2}];")
        lines.append("    }")
    for k2 in range(r2):
        lines.append(f"    {{ cplx<T> w[{r1}];")
        for n1 in range(r1):
            lines.append(f"      w[{n1}] = t[{n1 * r2 + k2}];")
        lines.append(f"      dft{r1}<T>(w);")
        for k1 in range(r1):
            lines.append(f"      v[{k2 + r2 * k1}] = w[{k1}];")
        lines.append("    }")
    lines.append("}")
    return lines


# Packed f32 arithmetic on sm_100+ (PTX add / sub / mul / fma .rn.f32x2): each lane rounds
# exactly as the scalar operation does.  A complex point is one register pair (x, y).
F32X2_HELPERS = [
    "#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000",
    "#define B200FFT_F32X2 1",
    "namespace f32x2 {",
    "using u64 = unsigned long long;",
    "__device__ __forceinline__ u64 pk(float x, float y) { u64 r; asm(\"mov.b64 %0, {%1, %2};\" : \"=l\"(r) : \"f\"(x), \"f\"(y)); return r; }",
    "__device__ __forceinline__ void up(u64 r, float &x, float &y) { asm(\"mov.b64 {%0, %1}, %2;\" : \"=f\"(x), \"=f\"(y) : \"l\"(r)); }",
    "__device__ __forceinline__ u64 add(u64 a, u64 b) { u64 r; asm(\"add.rn.f32x2 %0, %1, %2;\" : \"=l\"(r) : \"l\"(a), \"l\"(b)); return r; }",
    "__device__ __forceinline__ u64 sub(u64 a, u64 b) { u64 r; asm(\"sub.rn.f32x2 %0, %1, %2;\" : \"=l\"(r) : \"l\"(a), \"l\"(b)); return r; }",
    "__device__ __forceinline__ u64 mul(u64 a, u64 b) { u64 r; asm(\"mul.rn.f32x2 %0, %1, %2;\" : \"=l\"(r) : \"l\"(a), \"l\"(b)); return r; }",
    "// a * b + c",
    "__device__ __forceinline__ u64 fma(u64 a, u64 b, u64 c) { u64 r; asm(\"fma.rn.f32x2 %0, %1, %2, %3;\" : \"=l\"(r) : \"l\"(a), \"l\"(b), \"l\"(c)); return r; }",
    "}  // namespace f32x2",
    "#endif",
    "",
]

# f32 radix-2 butterfly: both complex sums in one packed add and one packed subtract (every
# larger power-of-two codelet is built from this butterfly).
F32X2_DFT2 = [
    "",
    "template <> B200FFT_HD void dft2<float>(cplx<float>* v) {",
    "#ifdef B200FFT_F32X2",
    "    const f32x2::u64 a = f32x2::pk(v[0].x, v[0].y), b = f32x2::pk(v[1].x, v[1].y);",
    "    f32x2::up(f32x2::add(a, b), v[0].x, v[0].y);",
    "    f32x2::up(f32x2::sub(a, b), v[1].x, v[1].y);",
    "#else",
    "    const cplx<float> a = v[0], b = v[1];",
    "    v[0].x = a.x + b.x; v[0].y = a.y + b.y;",
    "    v[1].x = a.x - b.x; v[1].y = a.y - b.y;",
    "#endif",
    "}",
]


# Primes whose f32 butterfly is packed.  Radix 7 measured slower packed (the fused 4099
# Bluestein line, M = 8 * 3 * 7^3: 4.30 -> 4.39 ms; its nine constant pairs per kind cost
# registers), so 7, 11 and 13 stay scalar.
F32X2_PRIMES = (2, 3, 5)


def emit_prime_f32x2(r):
    """f32 prime-radix butterfly on packed pairs: s_n = v_n + v_(r-n) packed; the
    differences are formed swapped, e_n = (dy, dx), so that b' = sum (s_nk, -s_nk) * e_n
    is (by, -bx) and the outputs v_k = a + b', v_(r-k) = a - b' are packed too, with
    a = x0 + sum c_nk s_n.  Lane by lane the operations of the scalar codelet."""
    h = (r - 1) // 2
    L = ["", f"template <> B200FFT_HD void dft{r}<float>(cplx<float>* v) {{", "#ifdef B200FFT_F32X2",
         "    using namespace f32x2;", "    const u64 x0 = pk(v[0].x, v[0].y);"]
    for n in range(1, h + 1):
        L.append(f"    const u64 s{n} = add(pk(v[{n}].x, v[{n}].y), pk(v[{r - n}].x, v[{r - n}].y));")
        L.append(f"    const u64 e{n} = pk(v[{n}].y - v[{r - n}].y, v[{n}].x - v[{r - n}].x);")
    acc = "x0"
    for n in range(1, h + 1):
        acc = f"add({acc}, s{n})"
    L.append(f"    up({acc}, v[0].x, v[0].y);")
    for k in range(1, h + 1):
        a = "x0"
        b = None
        for n in range(1, h + 1):
            c, sn = cs(n * k, r)
            cf, sf = lit(c).replace("kc<T>", "kc<float>"), lit(sn).replace("kc<T>", "kc<float>")
            a = f"fma(pk({cf}, {cf}), s{n}, {a})"
            term = f"pk({sf}, -{sf})"
            b = f"mul({term}, e{n})" if b is None else f"fma({term}, e{n}, {b})"
        L.append(f"    {{ const u64 a = {a};")
        L.append(f"      const u64 b = {b};")
        L.append(f"      up(add(a, b), v[{k}].x, v[{k}].y);")
        L.append(f"      up(sub(a, b), v[{r - k}].x, v[{r - k}].y); }}")
    L.append("#else")
    body = emit_prime(r)[1:-1]  # the generic body, specialised to float
    L.extend(line.replace("const T ", "const float ").replace("cplx<T>", "cplx<float>").replace("kc<T>", "kc<float>")
             for line in body)
    L.append("#endif")
    L.append("}")
    return L


def main():
    out = [
        "// Generated by gen_codelets.py -- do not edit by hand.",
        "// Forward DFT butterflies y[k] = sum_n v[n] exp(-2 pi i n k / R), in place.",
        "#pragma once",
        "",
        "#ifndef B200FFT_HD",
        "#ifdef __CUDACC__",
        "#define B200FFT_HD __host__ __device__ __forceinline__",
        "#else",
        "#define B200FFT_HD inline",
        "#endif",
        "#endif",
        "",
        "template <typename T> struct alignas(2 * sizeof(T)) cplx { T x, y; };",
        "",
        "// A constant of the butterflies: hi + lo with hi the nearest double (the value the",
        "// f32 / f64 codelets use) and lo the residual (used by the double-double type).",
        "template <typename T> struct KConst {",
        "    static B200FFT_HD T make(double hi, double) { return T(hi); }",
        "};",
        "template <typename T> B200FFT_HD T kc(double hi, double lo) { return KConst<T>::make(hi, lo); }",
        "",
    ] + F32X2_HELPERS
    done = set()

    def gen(r):
        if r in done:
            return
        if r in PRIMES:
            out.extend(emit_prime(r))
            if r in F32X2_PRIMES:
                out.extend(F32X2_DFT2 if r == 2 else emit_prime_f32x2(r))
        else:
            r1, r2 = SPLITS[r]
            gen(r1)
            gen(r2)
            out.extend(emit_split(r))
        out.append("")
        done.add(r)

    for r in RADICES:
        gen(r)
    out.append("template <int R, typename T> B200FFT_HD void dft(cplx<T>* v) {")
    for i, r in enumerate(RADICES):
        kw = "if" if i == 0 else "else if"
        out.append(f"    {kw} constexpr (R == {r}) dft{r}<T>(v);")
    out.append("}")
    path = os.path.join(HERE, "dft_codelets.cuh")
    with open(path, "w") as fh:
        fh.write("\n".join(out) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    main()
