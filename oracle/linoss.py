"""Oracle for the LinOSS scan and layer (test infrastructure; see ``oracle/__init__.py``).

Restates models/linoss/linoss.py of the reference: the sequential recurrence (155-180),
the three discretisations (183-232), the parameter constraints of ``LinOSS.forward``
(81-116) and the readout (118-120). Works in any floating dtype on the CPU.
"""
from __future__ import annotations

import torch


def linoss_recurrence(M11, M12, M21, M22, F1, F2):
    """[y1; y2]_t = M [y1; y2]_{t-1} + [F1; F2]_t from zero; returns the y2 trajectory.

    Restates ``_linoss_recurrence`` (models/linoss/linoss.py:171-180).
    """
    B, T, N = F1.shape
    y1 = F1.new_zeros(B, N)
    y2 = F2.new_zeros(B, N)
    outs = []
    for t in range(T):
        n1 = M11 * y1 + M12 * y2 + F1[:, t]
        n2 = M21 * y1 + M22 * y2 + F2[:, t]
        y1, y2 = n1, n2
        outs.append(y2)
    if not outs:
        return F2.new_zeros(B, 0, N)
    return torch.stack(outs, dim=1)


def discretise(variant: str, step, A, G=None):
    """(M11, M12, M21, M22, f1, f2) with F1 = f1 * Bu, F2 = f2 * Bu.

    variant "IM": models/linoss/linoss.py:189-196; "IMEX": 206-212;
    "DAMPED_IMEX": 223-231.
    """
    if variant == "IM":
        schur = 1.0 / (1.0 + step**2 * A)
        M11 = 1.0 - step**2 * A * schur
        M12 = -step * A * schur
        M21 = step * schur
        M22 = schur
        return M11, M12, M21, M22, M11 * step, M21 * step
    if variant == "IMEX":
        M11 = torch.ones_like(A)
        M12 = -step * A
        M21 = step
        M22 = 1.0 - step**2 * A
        return M11, M12, M21, M22, step, step**2
    if variant == "DAMPED_IMEX":
        S = 1.0 + step * G
        inv_S = 1.0 / S
        M11 = inv_S
        M12 = -step * inv_S * A
        M21 = step * inv_S
        M22 = 1.0 - step**2 * inv_S * A
        return M11, M12, M21, M22, step * inv_S, step**2 * inv_S
    raise ValueError(variant)


def constrain(variant: str, steps_raw, A_raw, G_raw=None, a_from_g: bool = True):
    """(step, A, G) after the constraints of ``LinOSS.forward`` (linoss.py:82-116)."""
    step = torch.sigmoid(steps_raw)
    if variant in ("IM", "IMEX"):
        return step, torch.relu(A_raw), None
    if a_from_g:
        G = torch.relu(G_raw)
        sqrt_term = torch.sqrt(1.0 + step * G)
        A_low = (2.0 + step * G - 2.0 * sqrt_term) / step**2
        A_high = (2.0 + step * G + 2.0 * sqrt_term) / step**2
        A = A_low + torch.relu(A_raw - A_low) - torch.relu(A_raw - A_high)
    else:
        A = torch.relu(A_raw)
        G_low = torch.relu(step * A - 2 * torch.sqrt(A))
        G_high = step * A + 2 * torch.sqrt(A)
        G = torch.clamp(G_raw, min=G_low, max=G_high)
    return step, A, G


def variant_name(discretization: str, damping: bool) -> str:
    if discretization == "IM":
        return "IM"
    return "DAMPED_IMEX" if damping else "IMEX"


def linoss_scan_fused(variant: str, steps_raw, A_raw, G_raw, Bu, a_from_g: bool = True):
    """Bu (S,L,P) complex -> y2 (S,L,P) complex: constraints + discretisation + recurrence.

    The composition LinOSS.forward performs between ``_project_input`` and the readout
    (models/linoss/linoss.py:82-116 with 183-232 and 155-180).
    """
    step, A, G = constrain(variant, steps_raw, A_raw, G_raw, a_from_g)
    M11, M12, M21, M22, f1, f2 = discretise(variant, step, A, G)
    return linoss_recurrence(M11, M12, M21, M22, f1 * Bu, f2 * Bu)


def project_input(B_param, x):
    """Bu = B x with complex B (P, H) from B_param (P, H, 2) (linoss.py:84, 148-152)."""
    B_complex = torch.complex(B_param[..., 0], B_param[..., 1])
    re = torch.einsum("nf,btf->btn", B_complex.real, x)
    im = torch.einsum("nf,btf->btn", B_complex.imag, x)
    return torch.complex(re, im)


def linoss_forward(params: dict, x, discretization="IMEX", damping=True, a_from_g=True):
    """Full layer forward (models/linoss/linoss.py:81-120) from a parameter dict with the
    reference's names: steps, A_diag, G_diag (damped only), B, C, D."""
    variant = variant_name(discretization, damping)
    Bu = project_input(params["B"], x)
    ys = linoss_scan_fused(
        variant, params["steps"], params["A_diag"], params.get("G_diag"), Bu, a_from_g
    )
    C_complex = torch.complex(params["C"][..., 0], params["C"][..., 1])
    Cy = torch.einsum("fn,btn->btf", C_complex, ys).real
    return Cy + x * params["D"]
