"""Answer extraction and equivalence for math rewards.

Role of the reference's ``env/parse_utils_qwen.py`` (answer extraction,
``strip_string`` normalisation) and ``env/grader.py`` (``math_equal``: string,
multiple-choice, numeric with percentage variants and a relative tolerance,
then symbolic equality under a timeout).  Written from the definitions, with
sympy for the symbolic step.
"""

from __future__ import annotations

import math
import re
import threading
from typing import Optional, Union

_BOXED = ("\\boxed", "\\fbox")
_NUMBER = re.compile(r"-?\d[\d,]*(?:\.\d+)?(?:e[-+]?\d+)?|-?\.\d+")


def last_boxed(text: str) -> Optional[str]:
    """Content of the last \\boxed{...} (balanced braces) or \\boxed x."""
    text = text or ""
    pos = max(text.rfind(b) for b in _BOXED)
    if pos < 0:
        return None
    i = pos
    while i < len(text) and text[i] not in "{ ":
        i += 1
    if i >= len(text):
        return None
    if text[i] == " ":
        m = re.match(r"\s*([^\s$]+)", text[i:])
        return m.group(1) if m else None
    depth, start = 0, i
    for j in range(i, len(text)):
        if text[j] == "{":
            depth += 1
        elif text[j] == "}":
            depth -= 1
            if depth == 0:
                return text[start + 1:j]
    return None


def _fix_fracs(s: str) -> str:
    # \frac12 -> \frac{1}{2}, \frac1{b} -> \frac{1}{b}
    out, i = [], 0
    while i < len(s):
        if s.startswith("\\frac", i):
            out.append("\\frac")
            i += 5
            for _ in range(2):
                if i < len(s) and s[i] == "{":
                    depth, j = 0, i
                    while j < len(s):
                        depth += s[j] == "{"
                        depth -= s[j] == "}"
                        if depth == 0:
                            break
                        j += 1
                    out.append(s[i:j + 1])
                    i = j + 1
                elif i < len(s):
                    out.append("{" + s[i] + "}")
                    i += 1
        else:
            out.append(s[i])
            i += 1
    return "".join(out)


def normalize(ans: str) -> str:
    """Canonical string form of an answer (LaTeX noise, units, spacing removed)."""
    s = str(ans or "").strip()
    s = s.replace("\n", "").rstrip(".")
    s = re.sub(r"\\text\{\s*([^}]*)\}", r"\1", s)
    for a, b in (("\\!", ""), ("\\,", ""), ("\\;", ""), ("\\left", ""), ("\\right", ""), ("dfrac", "frac"),
                 ("tfrac", "frac"), ("^{\\circ}", ""), ("^\\circ", ""), ("\\$", ""), ("$", ""), ("\\%", ""),
                 ("%", ""), ("\\displaystyle", "")):
        s = s.replace(a, b)
    s = re.sub(r"(\\mbox|\\mathrm)\{([^}]*)\}", r"\2", s)
    s = re.sub(r"\s*(units?|degrees?|cm|meters?|inches|feet|dollars?)\s*$", "", s)
    if "=" in s and len(s.split("=")[0].strip()) <= 2:
        s = s.split("=", 1)[1]
    s = re.sub(r"\\sqrt(\w)", r"\\sqrt{\1}", s)
    s = s.replace(" ", "")
    s = _fix_fracs(s)
    if re.fullmatch(r"-?\d+/\d+", s):
        a, b = s.split("/")
        s = f"\\frac{{{a}}}{{{b}}}"
    if s.startswith("."):
        s = "0" + s
    s = re.sub(r"(\d),(?=\d{3}(\D|$))", r"\1", s)
    if re.fullmatch(r"-?\d+\.0+", s):
        s = s.split(".")[0]
    return s


def extract_answer(text: str, data_name: str = "math", use_last_number: bool = True) -> str:
    text = text or ""
    boxed = last_boxed(text)
    if boxed is not None:
        return normalize(boxed)
    m = re.findall(r"(?:final answer|the answer) is[:\s]*\$?([^\n$]+)", text, re.IGNORECASE)
    if m:
        return normalize(m[-1])
    if data_name in ("mmlu", "gpqa", "choice"):
        c = re.findall(r"\b([A-E])\b", text)
        if c:
            return c[-1]
    if use_last_number:
        nums = _NUMBER.findall(text.replace("$", ""))
        if nums:
            return normalize(nums[-1])
    return ""


def _to_float(s: str) -> Optional[float]:
    s = str(s).replace(",", "").strip()
    m = re.fullmatch(r"\\frac\{(-?[\d.]+)\}\{(-?[\d.]+)\}", s)
    try:
        if m:
            return float(m.group(1)) / float(m.group(2))
        if s.endswith("%"):
            return float(s[:-1]) / 100
        return float(s)
    except (ValueError, ZeroDivisionError):
        return None


def numeric_equal(a: float, b: float, rel: float = 1e-4) -> bool:
    return math.isclose(a, b, rel_tol=rel, abs_tol=1e-9)


def _latex_to_sympy_text(s: str) -> str:
    s = re.sub(r"\\frac\{([^{}]*)\}\{([^{}]*)\}", r"((\1)/(\2))", s)
    s = re.sub(r"\\sqrt\{([^{}]*)\}", r"sqrt(\1)", s)
    s = s.replace("\\pi", "pi").replace("\\cdot", "*").replace("\\times", "*").replace("^", "**")
    s = s.replace("{", "(").replace("}", ")").replace("\\", "")
    return s


def _symbolic_equal(a: str, b: str) -> bool:
    import sympy
    from sympy.parsing.sympy_parser import (implicit_multiplication_application, parse_expr,
                                            standard_transformations)

    tr = standard_transformations + (implicit_multiplication_application,)
    ea = parse_expr(_latex_to_sympy_text(a), transformations=tr, evaluate=True)
    eb = parse_expr(_latex_to_sympy_text(b), transformations=tr, evaluate=True)
    if sympy.simplify(ea - eb) == 0:
        return True
    try:
        return numeric_equal(float(sympy.N(ea)), float(sympy.N(eb)))
    except (TypeError, ValueError):
        return False


def _with_timeout(fn, timeout_s: float, *args) -> bool:
    box = {}

    def run():
        try:
            box["v"] = bool(fn(*args))
        except Exception:  # noqa: BLE001 - unparsable means "not equal"
            box["v"] = False

    t = threading.Thread(target=run, daemon=True)
    t.start()
    t.join(timeout_s)
    return box.get("v", False)


def math_equal(prediction: Union[str, float, None], reference: Union[str, float, None], include_percentage: bool = True,
               timeout: bool = True, timeout_s: float = 3.0) -> bool:
    if prediction is None or reference is None:
        return False
    p, r = str(prediction).strip(), str(reference).strip()
    if p.lower() == r.lower():
        return True
    if r in ("A", "B", "C", "D", "E"):
        m = re.findall(r"[A-E]", p.upper())
        return bool(m) and m[-1] == r
    pn, rn = normalize(p), normalize(r)
    if pn == rn:
        return True
    pf, rf = _to_float(pn), _to_float(rn)
    if pf is not None and rf is not None:
        cands = [rf, rf / 100, rf * 100] if include_percentage else [rf]
        return any(numeric_equal(pf, c) for c in cands)
    if not pn:
        return False
    if (pn[:1] in "([" and pn[-1:] in ")]") and (rn[:1] in "([" and rn[-1:] in ")]"):
        pp, rr = pn[1:-1].split(","), rn[1:-1].split(",")
        return len(pp) == len(rr) and all(math_equal(x, y, include_percentage, timeout, timeout_s)
                                          for x, y in zip(pp, rr))
    if timeout:
        return _with_timeout(_symbolic_equal, timeout_s, pn, rn)
    try:
        return _symbolic_equal(pn, rn)
    except Exception:  # noqa: BLE001
        return False
