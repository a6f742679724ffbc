"""The soft backward's per-interval records, checked on the CPU.

Inside interval j (centres lo = c_{j-1}, hi = c_j, span S) the reference's
per-value gradient (docs/derivation.md of kapitan05/ace-kernels; restated in
src/ace_kernels/impls/v2_autograd.py:88-118)

    gp = g (coef_l (lw - (p - y - d_l) / S) + coef_r (rw + (p - y - d_r) / S)),
    rw = (p - lo) / S,  lw = 1 - rw,

is affine in p and y. The gradient kernel stores one record {F, D} per row and
interval and computes gp = F + D (2 p - y); these tests check that algebra in
float64, and that the two end intervals (both sides the same bin) reduce to
g coef.
"""

import torch


def reference_gp(g, cl, cr, dl, dr, lo, hi, p, y):  # type: ignore[no-untyped-def]
    s = hi - lo
    rw = (p - lo) / s
    lw = 1.0 - rw
    return g * (cl * (lw - (p - y - dl) / s) + cr * (rw + (p - y - dr) / s))


def record(g, cl, cr, dl, dr, lo, hi):  # type: ignore[no-untyped-def]
    """{F, D} as the gradient kernel's prologue builds them."""
    a, b = g * cl, g * cr
    inv = 1.0 / (hi - lo)
    d = (b - a) * inv
    e = inv * (a * dl - b * dr)
    return a - d * lo + e, d


def test_affine_record_equals_the_reference_formula() -> None:
    gen = torch.Generator().manual_seed(0)
    n = 100000
    k = 20
    j = torch.randint(1, k, (n,), generator=gen).double()
    lo, hi = (j - 0.5) / k, (j + 0.5) / k
    p = lo + (hi - lo) * torch.rand(n, generator=gen, dtype=torch.float64)
    y = (torch.rand(n, generator=gen) < 0.3).double()
    g = torch.rand(n, generator=gen, dtype=torch.float64)
    cl, cr = (torch.randn(2, n, generator=gen, dtype=torch.float64) * 1e-3).unbind(0)
    dl, dr = (torch.randn(2, n, generator=gen, dtype=torch.float64) * 0.1).unbind(0)
    f, d = record(g, cl, cr, dl, dr, lo, hi)
    got = f + d * (2.0 * p - y)
    want = reference_gp(g, cl, cr, dl, dr, lo, hi, p, y)
    scale = want.abs().max()
    assert ((got - want).abs().max() / scale).item() < 1e-12


def test_end_interval_record_is_g_coef() -> None:
    # both neighbours are the end bin: A = B, so D = 0 and F = g coef for any p, y
    g, c, dd = 0.7, 3e-4, -0.2
    t = lambda v: torch.tensor(v, dtype=torch.float64)  # noqa: E731
    f, d = record(t(g), t(c), t(c), t(dd), t(dd), t(0.0), t(1.0))
    assert d.item() == 0.0
    assert abs(f.item() - g * c) < 1e-18
