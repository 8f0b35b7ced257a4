"""TEST INFRASTRUCTURE ONLY: builds `oracle/_ref/libmlx_qmv_emu.so`, the reference's own Metal qmv
kernel source compiled for the CPU, used to pin the C restatement in `oracle/qmv_oracle.c`.

The reference keeps its kernels as Python string constants (IronMule ironmule/qmv_k3840.py:62-244,
ironmule/qmv_shared.py:30-138, ironmule/qmv_fast_shared.py:30-131, ironmule/qmv_variant.py:81-96). Those
modules import MLX at the top, which is absent here, so they are not imported: this script reads the files
with `ast`, evaluates only the module-level constants and the string-building functions (`_source`), and
formats the bodies exactly as the reference's `_kernel` / `kernel_for` do. The Metal text is compiled
unchanged under a C++ shim header that supplies what Metal and MLX's `metal_kernel` wrapper would:
address-space qualifiers (`device`, `thread` -> nothing), `uint3`, a `bfloat` type, `simd_sum` and the
kernel signature. Lanes of a SIMD group run one after another, lane 31 first, so that by the time lane 0
(the only lane that stores) calls `simd_sum`, every lane has deposited its value; `simd_sum` then reduces
with the xor butterfly the restatement also uses.

`bfloat + bfloat` is the one semantic the source leaves to the platform. The shim is built twice:
BF16_PARTIALS=0 (the sum stays float) and BF16_PARTIALS=1 (each add rounds to bfloat, as MLX's software
bfloat struct does); the restatement exposes the same switch.

Run here only (the reference tree is not on the GPU box): `python oracle/build_ref.py`. Outputs go to
`oracle/_ref/` and nowhere else. Nothing in the product imports this.
"""
from __future__ import annotations

import ast
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
# the IronMule checkout: $IRONMULE_REFERENCE, else a directory named "reference" beside this repository
REF = Path(os.environ.get("IRONMULE_REFERENCE", HERE.parents[1] / "reference")) / "ironmule"


def _module_constants(path: Path) -> tuple[dict, ast.Module]:
    """Evaluate the module-level assignments whose values are literals, names, string concatenation,
    integer arithmetic and `str.replace` -- enough for the kernel text and its constants."""
    tree = ast.parse(path.read_text())
    env: dict = {}

    def ev(node):
        if isinstance(node, ast.Constant):
            return node.value
        if isinstance(node, ast.Name):
            return env[node.id]
        if isinstance(node, ast.BinOp):
            a, b = ev(node.left), ev(node.right)
            ops = {ast.Add: lambda: a + b, ast.Mult: lambda: a * b, ast.FloorDiv: lambda: a // b,
                   ast.Sub: lambda: a - b}
            return ops[type(node.op)]()
        if isinstance(node, ast.Tuple):
            return tuple(ev(e) for e in node.elts)
        if isinstance(node, ast.Dict):
            return {ev(k): ev(v) for k, v in zip(node.keys, node.values)}
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and node.func.attr == "replace"):
            return ev(node.func.value).replace(*[ev(a) for a in node.args])
        raise ValueError("not a constant")

    for stmt in tree.body:
        if isinstance(stmt, ast.Assign) and len(stmt.targets) == 1 and isinstance(stmt.targets[0], ast.Name):
            try:
                env[stmt.targets[0].id] = ev(stmt.value)
            except (ValueError, KeyError):
                pass
    return env, tree


def _function(tree: ast.Module, name: str, env: dict):
    """Compile one module-level function (string building only) against the module's constants."""
    for stmt in tree.body:
        if isinstance(stmt, ast.FunctionDef) and stmt.name == name:
            mod = ast.Module(body=[stmt], type_ignores=[])
            ns = dict(env)
            exec(compile(mod, str(name), "exec"), ns)  # noqa: S102 - the reference's own string builder
            return ns[name]
    raise KeyError(name)


def k3840_body(env: dict, fixed_k: int | None, simdgroups: int, results: int) -> str:
    """qmv_k3840._kernel / qmv_variant.kernel_for, formatted the same way."""
    if fixed_k is None:
        decl, loop, tail = "const int in_vec_size = shape[0];", env["RUNTIME_LOOP"], env["RUNTIME_TAIL"]
    else:
        decl = f"constexpr int in_vec_size = {fixed_k};"
        loop, tail = env["FIXED_LOOP"].replace("15", str(fixed_k // env["BLOCK_SIZE"])), ""
    return env["BODY"].format(
        num_simdgroups=simdgroups, results_per_simdgroup=results, pack_factor=env["PACK_FACTOR"],
        bytes_per_pack=env["BYTES_PER_PACK"], values_per_thread=env["VALUES_PER_THREAD"],
        block_size=env["BLOCK_SIZE"], group_size=env["GROUP_SIZE"],
        scale_step_per_thread=env["SCALE_STEP_PER_THREAD"], in_vec_size_decl=decl, main_loop=loop, tail=tail)


SHIM = r"""
#include <stdint.h>
#include <string.h>
#include <algorithm>
#define device
#define thread
#define METAL_FUNC inline
typedef uint32_t uint;
struct uint3 { uint x, y, z; };
static inline int min(int a, int b) { return a < b ? a : b; }
static inline int clamp(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static inline float bits_to_f(uint16_t h) { uint32_t u = ((uint32_t)h) << 16; float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t f_to_bits(float f) {
  uint32_t u; memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
struct bfloat {
  uint16_t bits;
  bfloat() : bits(0) {}
  bfloat(float f) : bits(f_to_bits(f)) {}
  operator float() const { return bits_to_f(bits); }
};
#if BF16_PARTIALS
static inline bfloat operator+(bfloat a, bfloat b) { return bfloat((float)a + (float)b); }
#else
static inline float operator+(bfloat a, bfloat b) { return (float)a + (float)b; }
#endif
static inline float operator+(float a, bfloat b) { return a + (float)b; }
#if BF16_PARTIALS
static inline bfloat operator+(bfloat a, float b) { return bfloat((float)a + b); }
#endif
static inline float operator/(bfloat a, float b) { return (float)a / b; }

/* simd_sum over a SIMD group whose lanes run one after another, lane 31 first. */
static float g_slots[64][32];
static int g_calls[32];
static int g_lane;
static inline float simd_sum(float v) {
  int c = g_calls[g_lane]++;
  g_slots[c][g_lane] = v;
  if (g_lane != 0) return v;
  float r[32];
  for (int l = 0; l < 32; l++) r[l] = g_slots[c][l];
  for (int off = 16; off > 0; off >>= 1) {
    float n[32];
    for (int l = 0; l < 32; l++) n[l] = r[l] + r[l ^ off];
    memcpy(r, n, sizeof(r));
  }
  return r[0];
}
"""


def _kernel_fn(name: str, header: str, body: str, inputs: list[str], outputs: list[str]) -> str:
    types = {"w": "const uint32_t*", "scales": "const bfloat*", "biases": "const bfloat*", "shape": "const int*"}
    params = [f"{types.get(n, 'const bfloat*')} {n}" for n in inputs] + [f"bfloat* {n}" for n in outputs]
    params += ["uint3 threadgroup_position_in_grid", "uint simdgroup_index_in_threadgroup",
               "uint thread_index_in_simdgroup"]
    return (f"namespace ns_{name} {{\n{header}\nstatic void kern({', '.join(params)}) {{\n{body}\n}}\n}}\n")


def _driver(name: str, simdgroups: int, rows_per_group: int, nvec: int) -> str:
    """extern "C" entry: runs the grid MLX dispatches, (1, ceil(N/rows_per_group), 1) threadgroups."""
    xs = ", ".join(f"(const bfloat*)(x + {v} * (size_t)K)" for v in range(nvec))
    ys = ", ".join(f"(bfloat*)(y + {v} * (size_t)N)" for v in range(nvec))
    return f"""
extern "C" int emu_{name}(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                          const uint16_t* x, uint16_t* y, int K, int N) {{
  int shape[2] = {{K, N}};
  int groups = (N + {rows_per_group} - 1) / {rows_per_group};
  for (int gy = 0; gy < groups; gy++) {{
    for (uint sg = 0; sg < {simdgroups}; sg++) {{
      memset(g_calls, 0, sizeof(g_calls));
      for (int lane = 31; lane >= 0; lane--) {{
        g_lane = lane;
        uint3 tid = {{0u, (uint)gy, 0u}};
        ns_{name}::kern(w, (const bfloat*)scales, (const bfloat*)biases, {xs}, shape, {ys}, tid, sg, (uint)lane);
      }}
    }}
  }}
  return 0;
}}
"""


def generate() -> str:
    k_env, _ = _module_constants(REF / "qmv_k3840.py")
    s_env, s_tree = _module_constants(REF / "qmv_shared.py")
    f_env, f_tree = _module_constants(REF / "qmv_fast_shared.py")
    v_env, _ = _module_constants(REF / "qmv_variant.py")
    parts = [SHIM]
    drivers = []
    one = (["w", "scales", "biases", "x", "shape"], ["out"])
    # qmv_port (runtime K, with tail) and qmv_k3840 (fixed K), geometry (2, 4): qmv_k3840.py:280-281
    for name, fixed in (("qmv_port", None), ("qmv_k3840", 3840)):
        parts.append(_kernel_fn(name, k_env["HEADER"], k3840_body(k_env, fixed, 2, 4), *one))
        drivers.append(_driver(name, 2, 8, 1))
    # qmv_variant geometry (4, 8): qmv_variant.py:45, 81-96
    sg, r = v_env["QUALIFIED_GEOMETRY"]
    parts.append(_kernel_fn("qmv_variant", k_env["HEADER"], k3840_body(k_env, 3840, sg, r), *one))
    drivers.append(_driver("qmv_variant", sg, sg * r, 1))
    # qmv_shared widths 1 and 2: qmv_shared.py:141-155
    src = _function(s_tree, "_source", s_env)
    for width in (1, 2):
        ins = ["w", "scales", "biases"] + [f"x{v}" for v in range(width)] + ["shape"]
        name = f"qmv_shared_x{width}"
        parts.append(_kernel_fn(name, s_env["HEADER"], src(width), ins, [f"out{v}" for v in range(width)]))
        drivers.append(_driver(name, 2, 8, width))
    # qmv_fast_shared K in (4096, 15360), widths 1 and 2: qmv_fast_shared.py:134-147
    fsrc = _function(f_tree, "_source", f_env)
    for k in f_env["SUPPORTED_K"]:
        for width in (1, 2):
            ins = ["w", "scales", "biases"] + [f"x{v}" for v in range(width)] + ["shape"]
            name = f"qmv_fast_k{k}_x{width}"
            parts.append(_kernel_fn(name, f_env["HEADER"], fsrc(k, width), ins, [f"out{v}" for v in range(width)]))
            drivers.append(_driver(name, 2, 8, width))
    return "\n".join(parts + drivers)


def build() -> list[Path]:
    if not REF.is_dir():
        raise FileNotFoundError(f"reference tree not found at {REF}")
    OUT.mkdir(parents=True, exist_ok=True)
    source = OUT / "mlx_qmv_emu.cpp"
    source.write_text(generate())
    built = []
    for flag in (0, 1):
        lib = OUT / f"libmlx_qmv_emu_bf{flag}.so"
        cmd = ["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-strict-aliasing", "-fPIC", "-shared",
               f"-DBF16_PARTIALS={flag}", "-w", str(source), "-o", str(lib)]
        subprocess.run(cmd, check=True)
        built.append(lib)
    return built


if __name__ == "__main__":
    for path in build():
        print(path)
    sys.exit(0)
