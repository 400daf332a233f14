"""Source rules the CUDA code keeps, checked on the CPU:

* every bulk copy has one destination CTA (each CTA loads its own tiles; the
  peer-memory kernels run on several GPUs, where a copy that fans out across a
  cluster is not allowed);
* none of the batched-memcpy entry points (copies are one cudaMemcpyAsync each);
* no trap instructions or device asserts (a failed wait sets an error word and
  returns instead);
* every spin loop in device code is a bounded wait (it reads %globaltimer).

The patterns are assembled from pieces so this file does not itself contain
the forms it looks for.
"""

import os
import re

from conftest import PKG, REPO

CSRC = os.path.join(PKG, "csrc")


def _sources():
    roots = [CSRC, os.path.join(REPO, "include")]
    for root in roots:
        for name in sorted(os.listdir(root)):
            if name.endswith((".cu", ".cuh", ".h")):
                path = os.path.join(root, name)
                yield path, open(path).read()


def _code(text):
    """Source without // and /* */ comments."""
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def test_bulk_copies_have_one_destination():
    mc = "multi" + "ca" + "st"
    for path, text in _sources():
        for line in _code(text).splitlines():
            if "cp.async.bulk" in line:
                assert mc not in line, f"{os.path.basename(path)}: {line.strip()}"


def test_no_batched_memcpy():
    copy = "Mem" + "cpy"
    batch = "Ba" + "tch" + "Async"
    names = [pre + copy + mid + batch for pre in ("cuda", "cu") for mid in ("", "3D")]
    for path, text in _sources():
        for n in names:
            assert n not in text, os.path.basename(path)
    for path in ("bench.py", "__graft_entry__.py"):
        text = open(os.path.join(REPO, path)).read()
        for n in names:
            assert n not in text, path


def test_no_traps_or_device_asserts():
    for path, text in _sources():
        code = _code(text)
        assert "__" + "trap" not in code, os.path.basename(path)
        assert not re.search(r"\btrap\s*;", code), os.path.basename(path)
        assert not re.search(r"(?<!static_)\bassert\s*\(", code), os.path.basename(path)


def test_device_spin_loops_are_bounded():
    """Every `while` loop in the kernel headers polls a flag or barrier; each
    one must read the global timer (the bounded-wait pattern)."""
    for path, text in _sources():
        if not path.endswith(".cuh"):
            continue
        code = _code(text)
        for m in re.finditer(r"\bwhile\s*\(", code):
            # the loop body: up to the matching closing brace of the next block
            start = code.find("{", m.end())
            depth, i = 0, start
            while i < len(code):
                depth += {"{": 1, "}": -1}.get(code[i], 0)
                if depth == 0:
                    break
                i += 1
            window = code[max(0, m.start() - 400):i]
            assert "global_ns()" in window or "kWaitLimitNs" in window or "timeout_ns" in window, \
                f"{os.path.basename(path)}: unbounded loop near {code[m.start():m.start() + 80]!r}"
