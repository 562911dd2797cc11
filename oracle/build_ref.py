"""ORACLE TEST INFRASTRUCTURE -- builds oracle/_ref/libnnref.so and libnnref_fma.so.

Recipe that compiles the reference's own kernel source
(Experts/NeuroNet_DNG/NeuroNet.cl) for the host CPU.  It reads the file where
it lies in the reference checkout, extracts the helper block
(NeuroNet.cl:1-420: defines, IsNaNOrInf, fActivation, Deactivation,
Local* reductions) and every in-scope kernel by name, rewrites the OpenCL C
spellings that C++ does not accept (vector literals, address-space
qualifiers, __local arrays), and compiles the result together with
oracle/ref_shim.h and oracle/ref_exec.cpp into oracle/_ref/libnnref.so.

Two builds of the same source: libnnref.so evaluates every a*b+c as a rounded
product and a rounded sum (-ffp-contract=off); libnnref_fma.so lets the
compiler contract them into fused multiply-adds, as OpenCL C allows by default
(the FP_CONTRACT pragma is ON unless a program turns it off) and as GPU
OpenCL compilers do.  Both are valid executions of the reference; the second
needs a host CPU with FMA instructions.

Nothing from the reference is committed: the rewritten source is written
only to oracle/_ref/ (git-ignored).  When the reference checkout is absent
(e.g. on a machine that only received the built files) the script exits
without doing anything.

Usage:  python oracle/build_ref.py --reference DIR [--force]
        (or NN_REFERENCE_DIR=DIR python oracle/build_ref.py)
"""
from __future__ import annotations

import argparse
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
CL_RELPATH = os.path.join("Experts", "NeuroNet_DNG", "NeuroNet.cl")

# Every kernel of the hot path (the in-scope subset of NeuroNet.cl).
KERNELS = [
    "FeedForward", "CalcOutputGradient", "CalcHiddenGradient",
    "UpdateWeightsMomentum", "UpdateWeightsAdam",
    "FeedForwardConv", "CalcHiddenGradientConv",
    "UpdateWeightsConvMomentum", "UpdateWeightsConvAdam",
    "AttentionScore", "AttentionOut", "SumMatrix", "AttentionInsideGradients",
    "Normalize", "NormalizeWeights", "ConcatenateBuffers", "DeconcatenateBuffers",
    "MHAttentionScore", "MHAttentionOut", "MHAttentionInsideGradients",
    "Dropout", "BatchFeedForward", "CalcHiddenGradientBatch",
    "UpdateBatchOptionsMomentum", "UpdateBatchOptionsAdam",
    "LSTM_FeedForward", "LSTM_ConcatenatedGradient", "LSTM_HiddenGradient",
    "LSTM_UpdateWeightsAdam",
    "SoftMax_FeedForward", "SoftMax_HiddenGradient", "SoftMax_OutputGradient",
    "SoftUpdate", "SoftUpdateAdam",
    "Transpose", "MH2AttentionOut", "MH2AttentionInsideGradients",
    "RevInFeedForward", "RevInHiddenGraddient", "Activation", "DeActivation",
    "Concat_FeedForward", "Concat_HiddenGradient", "Concat_UpdateWeightsMomentum", "Concat_UpdateWeightsAdam",
    "UpdateWeightsAdamMini", "UpdateWeightsConvAdamMini", "MatMult", "MatMultGrad",
    "FQF_Cosine", "FQF_Output", "FQF_OutputGradient", "FQF_QuantileGradient", "FQF_CosineGradient",
    "FQF_FractionGradient", "FQF_CosineGradientSRM", "FQF_DistributionTargetGradient",
    "FQF_MonotoneRearrange", "FQF_RearrangeGradient", "FQF_SRMForward", "FQF_SRMGradient",
    "SAC_AlphaLogProbs", "SAC_AlphaGradients", "SAC_OutputGradient", "SAC_CalcLogProbs",
    "MHFlashAttention", "MHFlashAttentionGrad", "FQF_Sample", "PatchCreate", "PatchHiddenGradient",
]


def _match_close(text: str, start: int, open_ch: str, close_ch: str) -> int:
    """Index just past the bracket that closes the one at text[start]."""
    depth = 0
    i = start
    while i < len(text):
        c = text[i]
        if c == open_ch:
            depth += 1
        elif c == close_ch:
            depth -= 1
            if depth == 0:
                return i + 1
        i += 1
    raise ValueError("unbalanced brackets")


def _strip_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def extract_kernel(src: str, name: str) -> tuple[str, str, str]:
    """Return (full kernel text, parameter list text, body text)."""
    m = re.search(r"__kernel\s+void\s+" + re.escape(name) + r"\s*\(", src)
    if not m:
        raise KeyError(name)
    p_open = m.end() - 1
    p_close = _match_close(src, p_open, "(", ")")
    b_open = src.index("{", p_close)
    b_close = _match_close(src, b_open, "{", "}")
    return src[m.start():b_close], src[p_open + 1:p_close - 1], src[b_open:b_close]


def rewrite(code: str) -> str:
    """OpenCL C spellings -> C++ (inside namespace ocl of ref_shim.h)."""
    # __local arrays declared in a body become per-work-group statics.
    code = re.sub(r"__local\s+(float4|float2|float|int|uint)\s+(\w+)\s*\[",
                  r"static thread_local \1 \2[", code)
    code = re.sub(r"\b__local\b", "", code)
    code = re.sub(r"\b__global\b", "", code)
    code = re.sub(r"\b__constant\b", "const", code)
    code = re.sub(r"\b__kernel\b", "", code)
    # vector literals (floatN)(a,b,...) -> floatN(a,b,...)
    code = re.sub(r"\(\s*(float[248])\s*\)\s*\(", r"\1(", code)
    # scalar-to-vector casts (floatN)expr -> floatN(expr)
    code = re.sub(r"\(\s*(float[248])\s*\)\s*([A-Za-z0-9_.]+)", r"\1(\2)", code)
    return code


def parse_params(params: str) -> list[tuple[str, str]]:
    """[(kind, name)] with kind in p (pointer), i (int), u (uint), f (float)."""
    params = _strip_comments(params)
    out = []
    for raw in params.split(","):
        p = " ".join(raw.replace("\n", " ").split())
        if not p:
            continue
        is_ptr = "*" in p
        name = re.findall(r"[A-Za-z_]\w*", p)[-1]
        toks = re.findall(r"[A-Za-z_]\w*", p)
        if is_ptr:
            kind = "p"
        elif "float" in toks:
            kind = "f"
        elif "uint" in toks or "unsigned" in toks:
            kind = "u"
        else:
            kind = "i"
        out.append((kind, name, p))
    return out


# Kernels whose work-groups write the same elements (LSTM_HiddenGradient writes
# column 0 of rows >= 1 from its weight loop and, in another work-group, from
# its bias loop): executed with work-groups in order on one thread, so that the
# later loop's value is the one kept.
SERIAL_KERNELS = {"LSTM_HiddenGradient"}

# Data races in the reference source that a GPU hides (the work-group of these
# helpers is a single SIMD wavefront, so every lane's load happens before any
# lane's store) but a sequential work-item executor exposes.  Each patch adds
# the one barrier that makes the GPU ordering explicit.
RACE_PATCHES = [
    # LocalSoftMax (NeuroNet.cl:392-408): every lane reads Temp[0] (the max
    # returned by LocalMax) and LocalSum then stores Temp[id] with no barrier
    # in between, so lane 0 may overwrite the max before lane 1 reads it.
    ("float max=LocalMax(value,loc,Temp);", "float max=LocalMax(value,loc,Temp);\n   BarrierLoc", 1),
    # The same read of Temp[0] at the end of LocalMax / LocalMin (NeuroNet.cl:214-284), LocalSum
    # and LocalSum4: a kernel that calls them back to back on one local array (MHFlashAttention,
    # NeuroNet.cl:16066-16177: LocalMax, LocalSum, then LocalSum4 per feature group, per key tile)
    # lets a lane store its next value before the others have read the result.
    ("   return(Temp[0]);\n", "   const float result_=Temp[0];\n   BarrierLoc\n   return(result_);\n", 2),
    ("   result=IsNaNOrInf(Temp[0],0);\n", "   result=IsNaNOrInf(Temp[0],0);\n   BarrierLoc\n", 1),
    ("   result=IsNaNOrInf4(Temp[0],0.0f);\n", "   result=IsNaNOrInf4(Temp[0],0.0f);\n   BarrierLoc\n", 1),
]


# Helper functions that NeuroNet.cl defines between kernels (after the first __kernel), needed by a
# kernel in the list above: (return type and name as written).
LATE_HELPERS = ["float SRMCumulative(", "float SRMDensity("]


def _late_helper(cl_text: str, head: str) -> str:
    start = cl_text.index("\n" + head) + 1
    brace = cl_text.index("{", start)
    return cl_text[start:_match_close(cl_text, brace, "{", "}")] + "\n"


def generate(cl_text: str) -> str:
    first = cl_text.index("__kernel")
    helpers = cl_text[:first] + "".join(_late_helper(cl_text, h) for h in LATE_HELPERS)
    for old, new, count in RACE_PATCHES:
        if helpers.count(old) != count:
            raise RuntimeError(f"race patch anchor not found {count} times: {old!r}")
        helpers = helpers.replace(old, new)
    parts = ["// GENERATED by oracle/build_ref.py from the reference NeuroNet.cl -- do not commit.",
             '#include "ref_shim.h"', "namespace ocl {", "#line 1 \"NeuroNet.cl\"",
             rewrite(helpers)]
    table = []
    for name in KERNELS:
        text, params, body = extract_kernel(cl_text, name)
        line = cl_text[:cl_text.index(text)].count("\n") + 1
        parts.append(f'#line {line} "NeuroNet.cl"')
        parts.append(rewrite(text))
        plist = parse_params(params)
        uses_barrier = int(bool(re.search(r"BarrierLoc|barrier\s*\(|Local(Sum|Max|Min|SoftMax|SoftMaxGrad|Sum4)\s*\(",
                                          body)))
        table.append((name, plist, uses_barrier))
    parts.append("}  // namespace ocl")
    for name, plist, _ in table:
        args = []
        for idx, (kind, pname, decl) in enumerate(plist):
            if kind == "p":
                base = "uint" if re.search(r"\buint\b", decl) else ("int" if re.search(r"\bint\b", decl) else "float")
                args.append(f"(ocl::{base} *)a[{idx}]" if base == "uint" else f"({base} *)a[{idx}]")
            elif kind == "f":
                args.append(f"*(const float *)a[{idx}]")
            elif kind == "u":
                args.append(f"*(const unsigned int *)a[{idx}]")
            else:
                args.append(f"*(const int *)a[{idx}]")
        parts.append(f"static void call_{name}(void **a) {{ ocl::{name}({', '.join(args)}); }}")
    parts.append("struct RefKernel { const char *name; void (*call)(void **); int uses_barrier; int nargs; "
                 "const char *argtypes; int serial; };")
    rows = []
    for name, plist, ub in table:
        types = "".join(k for k, _, _ in plist)
        rows.append(f'  {{"{name}", call_{name}, {ub}, {len(plist)}, "{types}", {int(name in SERIAL_KERNELS)}}},')
    parts.append('extern "C" const RefKernel nnref_table[] = {\n' + "\n".join(rows) + "\n};")
    parts.append(f'extern "C" const int nnref_table_size = {len(table)};')
    return "\n".join(parts) + "\n"


# output name -> floating-point contraction flags
VARIANTS = {"libnnref.so": ["-ffp-contract=off"], "libnnref_fma.so": ["-ffp-contract=fast", "-mfma"]}


def build(reference: str, force: bool = False) -> str | None:
    """Builds both variants; returns the path of libnnref.so (None without the reference
    checkout and without an earlier build)."""
    cl_path = os.path.join(reference, CL_RELPATH)
    lib = os.path.join(OUT_DIR, "libnnref.so")
    if not os.path.exists(cl_path):
        return lib if os.path.exists(lib) else None
    deps = [cl_path, __file__, os.path.join(HERE, "ref_shim.h"), os.path.join(HERE, "ref_exec.cpp")]
    newest = max(os.path.getmtime(d) for d in deps)
    todo = [name for name in VARIANTS
            if force or not os.path.exists(os.path.join(OUT_DIR, name))
            or os.path.getmtime(os.path.join(OUT_DIR, name)) < newest]
    if not todo:
        return lib
    os.makedirs(OUT_DIR, exist_ok=True)
    with open(cl_path, "r", encoding="utf-8", errors="replace") as f:
        cl_text = f.read()
    gen = os.path.join(OUT_DIR, "nn_ref_gen.cpp")
    with open(gen, "w") as f:
        f.write(generate(cl_text))
    for name in todo:
        out = os.path.join(OUT_DIR, name)
        cmd = ["g++", "-O2", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-w", "-fno-fast-math",
               *VARIANTS[name], "-I", HERE, gen, os.path.join(HERE, "ref_exec.cpp"), "-o", out + ".tmp"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NN_REFERENCE_DIR"),
                    help="root of the EAPrognoz/NN_in_Trading checkout (or set NN_REFERENCE_DIR)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference DIR or set NN_REFERENCE_DIR")
    lib = build(a.reference, a.force)
    print(lib or "reference checkout not found; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
