#!/usr/bin/env python3
"""Build the reference shaders as CPU C++ ("shader-as-C++" harness).

TEST INFRASTRUCTURE ONLY.  Reads the reference's GLSL compute shaders from
``<reference>/kernels/`` at build time, rewrites the few GLSL-only constructs
(layout qualifiers, buffer blocks, push constants, ``out`` parameters, float
literals) into C++17, wraps each shader in its own namespace with a loop over
work groups and invocations, and compiles the result into
``oracle/_ref/libvkref.so``.  Generated sources and the library live only in
``oracle/_ref/`` (git-ignored): nothing derived from the reference is
committed.  The library runs the reference's own shader arithmetic on the
CPU and is used to pin the C restatement in ``oracle/oracle.c`` and to make
the golden vectors in ``tests/golden/``.

Exported entry point per shader ``<name>``::

    void vkref_<name>(void **bindings, const void *push_constants,
                      unsigned gx, unsigned gy, unsigned gz);

``bindings[i]`` is the host pointer bound at ``binding = i``.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"

# The shaders on the quantised-linear path (kernels/*.glsl in the reference).
SHADERS = [
    "dequant_q4_0", "dequant_q4_1", "dequant_q5_0", "dequant_q8_0", "dequant_q8_1",
    "dequant_q4_k", "dequant_q5_k", "dequant_q6_k",
    "linear_int8", "linear_fp16", "linear_fp16_fp32out",
    # the non-matmul kernels of the hipLaunchKernel table that need no
    # subgroup operations (rms_norm*.glsl and softmax_online.glsl reduce with
    # subgroup intrinsics, which this invocation-at-a-time harness cannot run)
    "elementwise_f32", "scale_f32", "binop_f32", "rope_neox", "embedding",
]

PRELUDE = r"""
// Generated prelude: GLSL scalar types and built-ins used by the shaders.
#include <cstdint>
#include <cstring>
#include <cmath>
#include <algorithm>
typedef uint32_t uint;
typedef _Float16 float16_t;
struct uvec3 { uint x, y, z; };
struct vec2 { float x, y; };
static inline vec2 unpackHalf2x16(uint v) {
    uint16_t lo = (uint16_t)(v & 0xFFFFu), hi = (uint16_t)(v >> 16);
    _Float16 a, b; std::memcpy(&a, &lo, 2); std::memcpy(&b, &hi, 2);
    return vec2{(float)a, (float)b};
}
template <class T> static inline T clamp(T v, T lo, T hi) { return v < lo ? lo : (v > hi ? hi : v); }
static inline float sign(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }
using std::abs; using std::exp; using std::max; using std::min; using std::round;
using std::tanh; using std::sqrt; using std::log; using std::pow; using std::cos; using std::sin;
"""

FLOAT_LIT = re.compile(r"(?<![\w.])((?:\d+\.\d*|\.\d+)(?:[eE][+-]?\d+)?)(?![\w.])")
BUF_RE = re.compile(
    r"layout\s*\(([^)]*)\)\s*(?:readonly|writeonly)?\s*(?:readonly|writeonly)?\s*buffer\s+(\w+)\s*"
    r"\{\s*([\w]+)\s+(\w+)\s*\[\s*\]\s*;\s*\}\s*(\w+)?\s*;", re.S)
PC_RE = re.compile(r"layout\s*\(\s*push_constant\s*\)\s*uniform\s+(\w+)\s*\{(.*?)\}\s*(\w+)\s*;", re.S)
LOCAL_RE = re.compile(r"layout\s*\(([^)]*local_size[^)]*)\)\s*in\s*;")


def translate(name: str, src: str) -> str:
    # Strip comments' effect on the regexes by keeping them (they are valid C++).
    lines = [l for l in src.splitlines() if not l.strip().startswith(("#version", "#extension"))]
    body = "\n".join(lines)

    m = LOCAL_RE.search(body)
    lx = ly = lz = 1
    if m:
        for part in m.group(1).split(","):
            k, v = [s.strip() for s in part.split("=")]
            if k == "local_size_x": lx = int(v)
            if k == "local_size_y": ly = int(v)
            if k == "local_size_z": lz = int(v)
        body = body[:m.start()] + body[m.end():]

    bindings = {}

    def buf_sub(mm):
        quals, _block, typ, member, inst = mm.groups()
        b = int(re.search(r"binding\s*=\s*(\d+)", quals).group(1))
        if inst:
            bindings[b] = f"{inst}.{member}"
            return f"static struct {{ {typ} *{member}; }} {inst};"
        bindings[b] = member
        return f"static {typ} *{member};"

    body = BUF_RE.sub(buf_sub, body)

    pc_type = None

    def pc_sub(mm):
        nonlocal pc_type
        pc_type = mm.group(1)
        return f"struct {mm.group(1)} {{{mm.group(2)}}};\nstatic {mm.group(1)} {mm.group(3)};"

    body = PC_RE.sub(pc_sub, body)
    body = re.sub(r"\bout\s+(float|int|uint)\s+(\w+)", r"\1 &\2", body)
    body = FLOAT_LIT.sub(lambda mm: mm.group(1) + "f", body)
    body = re.sub(r"\bvoid\s+main\s*\(\s*\)", "static void shader_main()", body)

    set_bufs = "\n".join(
        f"    {target} = ({ 'decltype(' + target + ')' }) bindings[{b}];" for b, target in sorted(bindings.items()))
    pc_copy = f"    std::memcpy(&pc, push, sizeof(pc));" if pc_type else ""
    return f"""
namespace {name} {{
static thread_local uvec3 gl_WorkGroupID, gl_LocalInvocationID, gl_GlobalInvocationID;
static const uvec3 gl_WorkGroupSize = {{{lx}u, {ly}u, {lz}u}};
{body}
}}  // namespace {name}

extern "C" void vkref_{name}(void **bindings, const void *push, unsigned gx, unsigned gy, unsigned gz) {{
    using namespace {name};
{set_bufs}
{pc_copy}
    long long total = (long long)gx * gy * gz;
#pragma omp parallel for schedule(static)
    for (long long g = 0; g < total; ++g) {{
        uvec3 wg{{(uint)(g % gx), (uint)((g / gx) % gy), (uint)(g / ((long long)gx * gy))}};
        for (uint z = 0; z < {lz}u; ++z)
        for (uint y = 0; y < {ly}u; ++y)
        for (uint x = 0; x < {lx}u; ++x) {{
            gl_WorkGroupID = wg;
            gl_LocalInvocationID = uvec3{{x, y, z}};
            gl_GlobalInvocationID = uvec3{{wg.x * {lx}u + x, wg.y * {ly}u + y, wg.z * {lz}u + z}};
            shader_main();
        }}
    }}
}}
"""


def main(reference: str | None = None) -> int:
    # $VKFLAME_REFERENCE, else a "reference" directory beside this repository
    ref = Path(reference or os.environ.get("VKFLAME_REFERENCE") or Path(__file__).resolve().parents[2] / "reference")
    kdir = ref / "kernels"
    if not kdir.is_dir():
        print(f"[build_ref] reference shaders not found at {kdir}; skipping", file=sys.stderr)
        return 1
    OUT.mkdir(parents=True, exist_ok=True)
    srcs = []
    for name in SHADERS:
        text = (kdir / f"{name}.glsl").read_text()
        cpp = OUT / f"gen_{name}.cpp"
        cpp.write_text(PRELUDE + translate(name, text))
        srcs.append(str(cpp))
    lib = OUT / "libvkref.so"
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-w", "-o", str(lib)] + srcs
    subprocess.run(cmd, check=True)
    print(f"[build_ref] built {lib}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else None))
