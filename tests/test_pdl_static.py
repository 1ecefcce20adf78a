"""
Every kernel the library launches with programmatic dependent launch (launch_pdl) must call
pdl_wait() before it touches memory another kernel writes, and in every block, or the kernels
after it could start before their inputs exist. A source check (no GPU): each kernel named in a
launch_pdl call has a body that calls pdl_wait(), and no early `return` comes before that call.
"""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "lazylora_b200", "csrc")


def _sources():
    out = {}
    for p in glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")):
        with open(p) as fh:
            out[p] = fh.read()
    return out


def _kernel_body(src, name):
    m = re.search(r"__global__[^;{]*?\b" + re.escape(name) + r"\s*\(", src, re.S)
    if not m:
        return None
    depth = 0
    # the body's opening brace follows the close of the parameter list
    k = m.end() - 1
    pd = 0
    while True:
        if src[k] == "(":
            pd += 1
        elif src[k] == ")":
            pd -= 1
            if pd == 0:
                break
        k += 1
    i = src.index("{", k)
    j = i
    while True:
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[i:j + 1]
        j += 1


def test_every_pdl_kernel_waits_first():
    srcs = _sources()
    allsrc = "\n".join(srcs.values())
    names = set()
    for m in re.finditer(r"launch_pdl\(\s*[^,]+,\s*([^,]+),", allsrc):
        names.update(re.findall(r"\b((?:k_|grouped_mxfp4_)\w+)", m.group(1)))
    # kernels picked through a local variable (auto kern = cond ? k_a<..> : k_b<..>)
    for m in re.finditer(r"auto\s+kern\s*=\s*([^;]+);", allsrc):
        names.update(re.findall(r"\b((?:k_|grouped_mxfp4_)\w+)", m.group(1)))
    assert len(names) >= 20, names
    missing = []
    for n in sorted(names):
        body = _kernel_body(allsrc, n)
        if body is None:
            missing.append(f"{n}: definition not found")
            continue
        w = body.find("pdl_wait()")
        if w < 0:
            missing.append(f"{n}: no pdl_wait()")
            continue
        r = body.find("return", 0, w)
        if r >= 0 and "pdl_wait" not in body[r - 200:r]:
            missing.append(f"{n}: returns before pdl_wait()")
    assert not missing, missing
