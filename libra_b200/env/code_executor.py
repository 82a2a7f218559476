"""Sandboxed code execution for code rewards and the code-agent tool.

Role of the reference's ``env/code_executor.py`` (local ``reliability_guard``
sandbox ``:114-190`` and remote SandboxFusion ``:577-960``).  Local mode runs
every test case in a fresh ``python -I`` subprocess: its own session, an empty
temporary working directory, a minimal environment, and rlimits on CPU time,
address space, file size and open files; a wall-clock timeout kills its process
group.  Two test formats:

* stdin/stdout: ``{"inputs": [str, ...], "outputs": [str, ...]}`` compared
  line by line after whitespace normalisation (numbers with a tolerance);
* function calls: ``{"fn_name": name, "inputs": [[args], ...], "outputs": [...]}``
  where the harness calls ``name(*args)`` and compares the JSON result.

Remote mode posts each case to a SandboxFusion ``/run_code`` endpoint.
"""

from __future__ import annotations

import asyncio
import json
import math
import os
import resource
import signal
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Dict, List, Optional, Tuple

DEFAULT_TIMEOUT = 10
DEFAULT_MEMORY_LIMIT_MB = 1024

_HARNESS = r"""
import json, sys
__ns = {"__name__": "__solution__"}
exec(compile(open(sys.argv[1]).read(), "solution.py", "exec"), __ns)
__args = json.loads(sys.stdin.read())
__fn = __ns.get(sys.argv[2])
if __fn is None and "Solution" in __ns:
    __fn = getattr(__ns["Solution"](), sys.argv[2])
__out = __fn(*__args) if isinstance(__args, list) else __fn(__args)
sys.stdout.write(json.dumps(__out, default=list))
"""


def run_sync(coro):
    """Run a coroutine from sync code, also when a loop is already running."""
    try:
        asyncio.get_running_loop()
    except RuntimeError:
        return asyncio.run(coro)
    with ThreadPoolExecutor(max_workers=1) as pool:
        return pool.submit(asyncio.run, coro).result()


def _limits(memory_mb: int, cpu_s: int):
    def apply():
        os.setsid()
        mem = memory_mb * 1024 * 1024
        resource.setrlimit(resource.RLIMIT_AS, (mem, mem))
        resource.setrlimit(resource.RLIMIT_CPU, (cpu_s, cpu_s + 1))
        resource.setrlimit(resource.RLIMIT_FSIZE, (16 << 20, 16 << 20))
        resource.setrlimit(resource.RLIMIT_NOFILE, (64, 64))
        resource.setrlimit(resource.RLIMIT_CORE, (0, 0))

    return apply


def _run_case(argv: List[str], stdin: str, cwd: str, timeout: float, memory_mb: int) -> Dict[str, Any]:
    env = {"PATH": "/usr/bin:/bin", "PYTHONHASHSEED": "0", "PYTHONDONTWRITEBYTECODE": "1", "HOME": cwd}
    p = subprocess.Popen(argv, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE, cwd=cwd,
                         env=env, preexec_fn=_limits(memory_mb, int(math.ceil(timeout)) + 1))
    try:
        out, err = p.communicate(stdin.encode(), timeout=timeout)
    except subprocess.TimeoutExpired:
        try:
            os.killpg(p.pid, signal.SIGKILL)  # the child leads its own session
        except ProcessLookupError:
            pass
        p.communicate()
        return {"status": "timeout", "stdout": "", "stderr": ""}
    return {"status": "success" if p.returncode == 0 else "runtime_error", "returncode": p.returncode,
            "stdout": out.decode(errors="replace"), "stderr": err.decode(errors="replace")[-2000:]}


def _same_output(got: str, want: str) -> bool:
    g = [ln.strip() for ln in got.strip().splitlines() if ln.strip()]
    w = [ln.strip() for ln in str(want).strip().splitlines() if ln.strip()]
    if g == w:
        return True
    if len(g) != len(w):
        return False
    for a, b in zip(g, w):
        ta, tb = a.split(), b.split()
        if len(ta) != len(tb):
            return False
        for x, y in zip(ta, tb):
            if x == y:
                continue
            try:
                if not math.isclose(float(x), float(y), rel_tol=1e-6, abs_tol=1e-6):
                    return False
            except ValueError:
                return False
    return True


def _same_value(got: Any, want: Any) -> bool:
    if isinstance(want, float) or isinstance(got, float):
        try:
            return math.isclose(float(got), float(want), rel_tol=1e-6, abs_tol=1e-6)
        except (TypeError, ValueError):
            return False
    if isinstance(want, (list, tuple)) and isinstance(got, (list, tuple)):
        return len(got) == len(want) and all(_same_value(a, b) for a, b in zip(got, want))
    return got == want


def local_check_correctness(test_cases: Dict[str, Any], code: str, timeout: float = DEFAULT_TIMEOUT,
                            memory_mb: int = DEFAULT_MEMORY_LIMIT_MB) -> Tuple[List[Any], List[Dict[str, Any]]]:
    inputs, outputs = list(test_cases.get("inputs") or []), list(test_cases.get("outputs") or [])
    fn = test_cases.get("fn_name")
    results, metas = [], []
    with tempfile.TemporaryDirectory(prefix="libra_sandbox_") as d:
        src = os.path.join(d, "solution.py")
        with open(src, "w", encoding="utf-8") as f:
            f.write(code)
        if fn:
            harness = os.path.join(d, "harness.py")
            with open(harness, "w", encoding="utf-8") as f:
                f.write(_HARNESS)
        for inp, want in zip(inputs, outputs):
            if fn:
                meta = _run_case([sys.executable, "-I", harness, src, str(fn)], json.dumps(inp), d, timeout, memory_mb)
                ok = False
                if meta["status"] == "success":
                    try:
                        ok = _same_value(json.loads(meta["stdout"]), want)
                    except ValueError:
                        ok = False
            else:
                meta = _run_case([sys.executable, "-I", src], str(inp), d, timeout, memory_mb)
                ok = meta["status"] == "success" and _same_output(meta["stdout"], want)
            results.append(ok if meta["status"] in ("success", "runtime_error") else -1)
            metas.append(meta)
    return results, metas


def remote_check_correctness(url: str, test_cases: Dict[str, Any], code: str, timeout: float = DEFAULT_TIMEOUT,
                             memory_mb: int = DEFAULT_MEMORY_LIMIT_MB, language: str = "python"):
    import requests

    inputs, outputs = list(test_cases.get("inputs") or []), list(test_cases.get("outputs") or [])
    results, metas = [], []
    for inp, want in zip(inputs, outputs):
        payload = {"code": code, "language": language, "stdin": str(inp), "run_timeout": timeout,
                   "memory_limit_MB": memory_mb}
        try:
            r = requests.post(url.rstrip("/") + "/run_code", json=payload, timeout=timeout + 30)
            body = r.json()
            run = body.get("run_result") or {}
            out = run.get("stdout", "")
            status = "success" if body.get("status") == "Success" and run.get("return_code", 1) == 0 else "error"
        except Exception as exc:  # noqa: BLE001 - reported per case
            out, status, body = "", "error", {"error": str(exc)}
        results.append(status == "success" and _same_output(out, want))
        metas.append({"status": status, "response": body})
    return results, metas


class CodeExecutor:
    def __init__(self, mode: str = "local", sandbox_fusion_url: Optional[str] = None, timeout: float = DEFAULT_TIMEOUT,
                 memory_limit_mb: int = DEFAULT_MEMORY_LIMIT_MB, language: str = "python", max_concurrency: int = 32):
        if mode not in ("local", "remote"):
            raise ValueError(f"mode must be 'local' or 'remote', got {mode}")
        if mode == "remote" and not sandbox_fusion_url:
            raise ValueError("sandbox_fusion_url is required when mode='remote'")
        self.mode, self.url, self.timeout = mode, sandbox_fusion_url, timeout
        self.memory_limit_mb, self.language = memory_limit_mb, language
        self._sem = asyncio.Semaphore(max_concurrency)

    async def execute(self, code: str, test_cases: Dict[str, Any]) -> Tuple[float, Dict[str, Any]]:
        loop = asyncio.get_running_loop()
        async with self._sem:
            if self.mode == "remote":
                results, metas = await loop.run_in_executor(None, remote_check_correctness, self.url, test_cases,
                                                            code, self.timeout, self.memory_limit_mb, self.language)
            else:
                results, metas = await loop.run_in_executor(None, local_check_correctness, test_cases, code,
                                                            self.timeout, self.memory_limit_mb)
        valid = [r for r in results if r is True or r is False]
        if not valid:
            return 0.0, {"error": "no test case ran to completion", "results": results, "metadata_list": metas}
        passed = sum(1 for r in valid if r)
        return passed / len(valid), {"pass_rate": passed / len(valid), "passed": passed, "total": len(valid),
                                     "results": results, "metadata_list": metas}

    async def run(self, code: str, stdin: str = "") -> Dict[str, Any]:
        """Execute once and return stdout/stderr (the code agent's tool)."""
        loop = asyncio.get_running_loop()
        with tempfile.TemporaryDirectory(prefix="libra_sandbox_") as d:
            src = os.path.join(d, "main.py")
            with open(src, "w", encoding="utf-8") as f:
                f.write(code)
            async with self._sem:
                return await loop.run_in_executor(None, _run_case, [sys.executable, "-I", src], stdin, d,
                                                  self.timeout, self.memory_limit_mb)

    @staticmethod
    def extract_code_block(text: str) -> Optional[str]:
        from libra_b200.env.rewards import extract_code_block

        return extract_code_block(text)
