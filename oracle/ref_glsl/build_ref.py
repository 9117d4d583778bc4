#!/usr/bin/env python
"""Compile AIHost's own attention shaders for the CPU (TEST INFRASTRUCTURE ONLY).

Reads the GLSL sources where they lie in the reference checkout — the inline strings of
AIHost/AIHost/Compute/ComputeShaders.cs, or the deployed file AIHost/Shaders/Vulkan/<name>.glsl
that ComputeShaders.TryLoadOrInline prefers (ComputeShaders.cs:73-85, ShaderLoader.cs:11-48) —
turns each into a C++ namespace with a light mechanical rewrite of the GLSL-only syntax
(buffer blocks -> pointers/structs, `shared` -> static, main -> main_), and builds
oracle/_ref/libref_glsl.so together with harness.cpp (the ComputeOps dispatch sequence) and
glsl_runtime.cpp. Nothing from the reference is copied into the repository: the generated
translation unit and the library live only in oracle/_ref/ (git-ignored).

Usage: python oracle/ref_glsl/build_ref.py [--reference PATH_TO_REFERENCE_CHECKOUT]
The checkout defaults to $AIHOST_REFERENCE_DIR, else a directory named `reference` beside this
repository's root.
"""
from __future__ import annotations

import argparse
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref"


def default_reference() -> Path:
    """$AIHOST_REFERENCE_DIR, else `reference` beside the repository root."""
    import os

    env = os.environ.get("AIHOST_REFERENCE_DIR")
    return Path(env) if env else HERE.parent.parent.parent / "reference"

# shader name used by TryLoadOrInline -> inline constant in ComputeShaders.cs (private const)
SHADERS = {
    "rope_full": "_inlineRoPEFull",
    "concat_axis0": "_inlineConcatAxis0",
    "fused_mha_generate": "_inlineFusedMHAGenerate",
    "matmul": "_inlineMatMul",
    "transpose": "_inlineTranspose",
    "scale": "_inlineScale",
    "causal_mask": "_inlineCausalMask",
    "rowwise_softmax": "_inlineRowwiseSoftmax",
    "slice_cols": "_inlineSliceCols",
    "scatter_cols": "_inlineScatterCols",
    "layernorm": "_inlineLayerNorm",
    "matmul_weights": "_inlineMatMulWeights",
}
# the K-quant dequantisation shaders: inline constants in QuantizationFormats.cs (public const),
# ComputeShaders.cs:12-16
QUANT_SHADERS = {f"dequant_q{k}k": f"DequantizeQ{k}K_Correct" for k in (2, 3, 4, 5, 6)}


def deployed_shaders(ref: Path) -> set[str]:
    """Vulkan shader files the reference copies next to its assembly (csproj Content items);
    ShaderLoader.Load (ShaderLoader.cs:11-48) finds only these, everything else falls back to
    the inline source (ComputeShaders.TryLoadOrInline, ComputeShaders.cs:73-85)."""
    proj = (ref / "AIHost/AIHost.csproj").read_text()
    return set(re.findall(r'Content Include="Shaders\\Vulkan\\(\w+)\.glsl"', proj))


BLOCK_RE = re.compile(
    r"layout\s*\(([^)]*)\)\s*((?:(?:readonly|writeonly|coherent|restrict|volatile)\s+)*)buffer\s+(\w+)\s*"
    r"\{([^}]*)\}\s*(\w*)\s*;", re.S)
LOCAL_RE = re.compile(r"layout\s*\(\s*local_size_x\s*=\s*(\d+)(?:\s*,\s*local_size_y\s*=\s*(\d+))?"
                      r"(?:\s*,\s*local_size_z\s*=\s*(\d+))?\s*\)\s*in\s*;")


def load_sources(ref: Path) -> dict[str, str]:
    cs = (ref / "AIHost/AIHost/Compute/ComputeShaders.cs").read_text()
    qf = (ref / "AIHost/AIHost/Compute/QuantizationFormats.cs").read_text()
    deployed = deployed_shaders(ref)
    out = {}
    for table, text, kind in ((SHADERS, cs, "private"), (QUANT_SHADERS, qf, "public")):
        for name, const in table.items():
            if name in deployed:
                out[name] = (ref / "AIHost/AIHost/Shaders/Vulkan" / f"{name}.glsl").read_text()
                continue
            m = re.search(kind + r" const string " + re.escape(const) + r'\s*=\s*@"(.*?)";', text, re.S)
            if not m:
                raise SystemExit(f"shader constant {const} not found")
            out[name] = m.group(1).replace('""', '"')
    return out


def translate(name: str, src: str) -> str:
    m = LOCAL_RE.search(src)
    if not m:
        raise SystemExit(f"{name}: no local_size layout")
    local = [int(m.group(i) or 1) for i in (1, 2, 3)]
    body = LOCAL_RE.sub("", src)
    body = re.sub(r"#version[^\n]*\n", "", body)
    binds = []
    decls = []

    def block(mb):
        layout, _quals, tname, members, inst = mb.groups()
        bm = re.search(r"binding\s*=\s*(\d+)", layout)
        binding = int(bm.group(1))
        fields = [f.strip() for f in members.split(";") if f.strip()]
        parsed = []
        for f in fields:
            fm = re.match(r"(\w+)\s+(\w+)\s*(\[\s*\])?$", f)
            if not fm:
                raise SystemExit(f"{name}: cannot parse block member '{f}'")
            parsed.append((fm.group(1), fm.group(2), bool(fm.group(3))))
        arrays = [p for p in parsed if p[2]]
        if arrays and len(parsed) != 1:
            raise SystemExit(f"{name}: mixed array/scalar block {tname}")
        if arrays:
            t, n, _ = arrays[0]
            if inst:
                decls.append(f"struct {tname}_blk {{ {t}* {n}; }};\nstatic {tname}_blk {inst};")
                binds.append(f"  if (binding == {binding}) {{ {inst}.{n} = static_cast<{t}*>(ptr); return; }}")
            else:
                decls.append(f"static {t}* {n};")
                binds.append(f"  if (binding == {binding}) {{ {n} = static_cast<{t}*>(ptr); return; }}")
        else:
            members_cpp = " ".join(f"{t} {n};" for t, n, _ in parsed)
            iname = inst or f"{tname}_anon"
            decls.append(f"struct {tname}_blk {{ {members_cpp} }};\nstatic {tname}_blk {iname};")
            if not inst:
                for t, n, _ in parsed:
                    decls.append(f"static {t}& {n} = {iname}.{n};")
            binds.append(f"  if (binding == {binding}) {{ std::memcpy(&{iname}, ptr, sizeof({iname})); return; }}")
        return ""

    body = BLOCK_RE.sub(block, body)
    body = re.sub(r"\bshared\s+", "static ", body)
    # GLSL `out` parameters become references
    body = re.sub(r"\bout\s+(float|uint|int)\s+(\w+)", r"\1& \2", body)
    if name.startswith("dequant_"):
        # GLSL float literals are single precision (here: 0.0, 32.0)
        body = re.sub(r"(?<![\w.])(\d+\.\d*(?:[eE][-+]?\d+)?)(?![\w.])", r"\1f", body)
    body = re.sub(r"\bvoid\s+main\s*\(\s*\)", "void main_()", body)
    uses_barrier = "barrier()" in body
    return (
        f"namespace sh_{name} {{\nusing namespace glsl;\n"
        f"static const uvec3 gl_WorkGroupSize = {{{local[0]}u, {local[1]}u, {local[2]}u}};\n"
        + "\n".join(decls) + "\n" + body +
        f"\nvoid bind(int binding, void* ptr) {{\n" + "\n".join(binds) + "\n}\n"
        f"void run(uint gx, uint gy, uint gz) {{ glsl::dispatch(main_, gl_WorkGroupSize, uvec3{{gx, gy, gz}}, "
        f"{'true' if uses_barrier else 'false'}); }}\n}}  // namespace sh_{name}\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(default_reference()))
    args = ap.parse_args()
    ref = Path(args.reference)
    if not (ref / "AIHost/AIHost/Compute/ComputeShaders.cs").exists():
        print("reference checkout not found; oracle/_ref not built", file=sys.stderr)
        return 1
    OUT.mkdir(exist_ok=True)
    srcs = load_sources(ref)
    tu = ['// GENERATED by oracle/ref_glsl/build_ref.py from the reference checkout; not part of the repository.',
          '#include "glsl_cpu.hpp"']
    tu += [translate(n, s) for n, s in srcs.items()]
    gen = OUT / "ref_shaders.cpp"
    gen.write_text("\n".join(tu))
    lib = OUT / "libref_glsl.so"
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    cmd = [cxx, "-std=c++20", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread",
           f"-I{HERE}", "-o", str(lib), str(gen), str(HERE / "glsl_runtime.cpp"), str(HERE / "harness.cpp")]
    subprocess.run(cmd, check=True)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
