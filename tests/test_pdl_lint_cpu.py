"""Programmatic dependent launch (PDL) ordering, checked on the sources.

Every kernel launched through ``launch_k`` carries the programmatic-stream-serialization
attribute: it may start as soon as the previous kernel on the stream has executed
``griddepcontrol.launch_dependents`` (``pdl_entry`` issues it right after its own wait).
The ordering of the whole chain rests on each such kernel executing
``griddepcontrol.wait`` (``pdl_wait`` / ``pdl_entry``) before it touches anything the
previous kernels wrote AND before it can exit: a kernel that returns without waiting
completes while its predecessor may still run, and the next kernel's wait then covers
only the early-finished one.  The fused all-reduce's parity argument (a peer runs at most
one reduction ahead) and the frozen workspaces of the captured decode step both depend on
that chain.  This test finds every PDL-launched kernel and checks that a wait comes
before its first ``return`` (through helper device functions too)."""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WAITS = {"pdl_wait", "pdl_entry"}


def _strip(t: str) -> str:
    t = re.sub(r"//[^\n]*", "", t)
    return re.sub(r"/\*.*?\*/", "", t, flags=re.S)


def _body(text: str, i: int) -> str:
    j = text.index("{", i)
    d = 0
    for k in range(j, len(text)):
        if text[k] == "{":
            d += 1
        elif text[k] == "}":
            d -= 1
            if d == 0:
                return text[j:k + 1]
    raise AssertionError("unbalanced braces")


def _sources():
    files = glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.cu")) + glob.glob(
        os.path.join(ROOT, "csrc", "kernels", "*.cuh"))
    return {os.path.basename(f): _strip(open(f).read()) for f in files}


def _waiters(allsrc: str) -> set:
    """Device functions that execute a PDL wait (transitively, three levels)."""
    w = set(WAITS)
    for _ in range(3):
        for m in re.finditer(r"(?:MOET_DEVICE|__device__)[^;{()]*?\b(\w+)\s*\(", allsrc):
            if m.group(1) in w:
                continue
            try:
                b = _body(allsrc, m.end())
            except ValueError:
                continue
            if any(re.search(r"\b%s\s*(<[^>]*>)?\s*\(" % x, b) for x in w):
                w.add(m.group(1))
    return w


def _pdl_launched(src: dict) -> set:
    names = set()
    for t in src.values():
        for m in re.finditer(r"launch_k\(\s*(\w+)", t):
            names.add(m.group(1))
        if "launch_k(kern" in t:     # a kernel chosen into a variable or a launch helper
            for m in re.finditer(r"\bkern\s*=\s*([^;]+);", t):
                names.update(re.findall(r"(\w+_kernel)\b", m.group(1)))
            for m in re.finditer(r"\blaunch\(\s*(\w+_kernel)\b", t):
                names.add(m.group(1))
    names.discard("kern")
    names.discard("void")         # the definition of launch_k itself
    return names


def test_every_pdl_launched_kernel_waits_before_it_can_exit():
    src = _sources()
    allsrc = "\n".join(src.values())
    waiters = _waiters(allsrc)
    launched = _pdl_launched(src)
    assert len(launched) >= 30, sorted(launched)       # the scan sees the decode step's kernels
    bad = []
    for name in sorted(launched):
        m = re.search(r"__global__[^;{]*?\b%s\s*\(" % name, allsrc)
        assert m, f"kernel {name} launched with launch_k but not defined"
        b = _body(allsrc, m.end())
        calls = [mm.start() for x in waiters for mm in re.finditer(r"\b%s\s*(<[^>]*>)?\s*\(" % x, b)]
        if not calls:
            bad.append(f"{name}: never waits")
            continue
        first = min(calls)
        early = [mm.start() for mm in re.finditer(r"\breturn\b", b) if mm.start() < first]
        if early:
            bad.append(f"{name}: returns before its PDL wait")
    assert not bad, bad


def test_lint_catches_an_early_exit():
    fake = {"k.cu": _strip("""
        MOET_DEVICE void helper() { pdl_entry(); }
        __global__ void good_kernel(int* p) { helper(); if (!p) return; *p = 1; }
        __global__ void bad_kernel(int* p) { if (!p) return; pdl_entry(); *p = 1; }
        void host() { launch_k(good_kernel, 1, 1, 0, 0, nullptr); launch_k(bad_kernel, 1, 1, 0, 0, nullptr); }
    """)}
    allsrc = fake["k.cu"]
    w = _waiters(allsrc)
    assert "helper" in w
    for name, ok in (("good_kernel", True), ("bad_kernel", False)):
        m = re.search(r"__global__[^;{]*?\b%s\s*\(" % name, allsrc)
        b = _body(allsrc, m.end())
        first = min(mm.start() for x in w for mm in re.finditer(r"\b%s\s*\(" % x, b))
        assert (not any(mm.start() < first for mm in re.finditer(r"\breturn\b", b))) == ok
    assert _pdl_launched(fake) == {"good_kernel", "bad_kernel"}
