"""Generate the golden vectors of the hot path by running the REFERENCE's own Triton kernels on the CPU.

Runs only where the ComfyUI-WeightFerry sources are available (pass --ref DIR; the tests never run this script and
never read the reference). Each kernel is loaded from its file, its @triton.jit closure helpers are made module
globals (the interpreter resolves them there) and it is launched under TRITON_INTERPRET=1 with the reference's own
launch arguments on small seeded inputs.

The interpreter cannot execute three hardware operations the kernels use; they are given their documented
semantics here (and nothing else of the kernels is changed):
  * inline PTX ``cvt.rn.f16.f32 t, $1; cvt.f32.f16 $0, t;`` -> round to the nearest float16 (ties to even) and back;
  * inline PTX ``rsqrt.approx.f32`` -> the correctly rounded float32 reciprocal square root (the hardware
    approximation is within 2 ulp of it; the fixtures that go through it are compared with a 2-ulp tolerance);
  * ``libdevice.rint`` -> round half to even; and the interpreter's ``fma``, which it evaluates as a product and a
    sum rounded separately, is replaced by a correctly rounded fused multiply-add.
Outputs: one .npz per kernel family in this folder (inputs and outputs, raw bits for 16-bit dtypes).

    python tests/golden/make_golden.py --ref /path/to/ComfyUI-WeightFerry
"""

import argparse
import importlib.util
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
SEED = 20261201


# ------------------------------------------------------------------------------------------- interpreter patches
def _fma_exact(x, y, z):
    """Correctly rounded float32 fma. The product is exact in float64; s = fl64(p + z) and its error e (TwoSum) give
    p + z = s + e exactly. Rounding s to float32 is right unless s lies exactly on a float32 midpoint with e != 0;
    then the exact sum is just off the midpoint, on the side of e."""
    x64, y64, z64 = (np.asarray(v, dtype=np.float64) for v in (x, y, z))
    p = x64 * y64
    s = p + z64
    bp = s - z64
    e = (p - bp) + (z64 - (s - bp))
    r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    toward = np.where(s > r64, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    other = np.nextafter(r, toward).astype(np.float64)
    is_mid = (s != r64) & (s == (r64 + other) / 2)
    go_other = is_mid & (np.sign(e) == np.sign(other - r64)) & (e != 0)
    return np.where(go_other, other, r64).astype(np.float32)


def _fma_exact_checked(x, y, z):
    """_fma_exact, cross-checked by exact rational arithmetic on a sample (guards the midpoint logic)."""
    out = _fma_exact(x, y, z)
    from fractions import Fraction
    xs, ys, zs, os_ = (np.asarray(v, np.float32).reshape(-1) for v in (x, y, z, out))
    for i in range(0, xs.size, max(1, xs.size // 64)):
        if not (np.isfinite(xs[i]) and np.isfinite(ys[i]) and np.isfinite(zs[i])):
            continue
        exact = Fraction(float(xs[i])) * Fraction(float(ys[i])) + Fraction(float(zs[i]))
        r = np.float32(float(exact))  # nearest double, then float32: double rounding possible only at midpoints
        cands = [np.nextafter(r, np.float32(-np.inf)), r, np.nextafter(r, np.float32(np.inf))]
        best = min(cands, key=lambda c: (abs(Fraction(float(c)) - exact),
                                        int(np.float32(c).view(np.uint32)) & 1))
        assert np.float32(best).view(np.uint32) == os_[i].view(np.uint32), (xs[i], ys[i], zs[i])
    return out


def patch_interpreter():
    from triton.runtime import interpreter as it
    B = it.InterpreterBuilder

    def create_inline_asm(self, inlineAsm, constraints, values, type, isPure, pack):
        asm = " ".join(inlineAsm.split())
        x = values[0].data
        if "cvt.rn.f16.f32" in asm:
            r = x.astype(np.float32).astype(np.float16).astype(np.float32)
        elif "rsqrt.approx.f32" in asm:
            r = (1.0 / np.sqrt(x.astype(np.float64))).astype(np.float32)
        else:
            raise NotImplementedError(asm)
        res = it.TensorHandle(r, values[0].dtype.scalar)
        return types.SimpleNamespace(get_result=lambda i: res)

    def create_extern_elementwise(self, libName, libPath, symbol, argList, retType, isPure):
        if "rint" in symbol:
            x = argList[0].data
            return it.TensorHandle(np.rint(x).astype(x.dtype), argList[0].dtype.scalar)
        raise NotImplementedError(symbol)

    def create_fma(self, x, y, z):
        return it.TensorHandle(_fma_exact_checked(x.data, y.data, z.data), z.dtype.scalar)

    # libdevice.rint outside the builder: the interpreter does not route tl.extra.cuda.libdevice through it
    import triton.language as tl
    from triton.language.extra.cuda import libdevice

    def rint(x, _semantic=None, **_kw):
        return tl.tensor(it.TensorHandle(np.rint(x.handle.data).astype(x.handle.data.dtype), x.handle.dtype), x.type)
    libdevice.rint = rint

    B.create_inline_asm = create_inline_asm
    B.create_extern_elementwise = create_extern_elementwise
    B.create_fma = create_fma


def load_ref(ref, rel, name):
    pkg = sys.modules.get("wfref")
    if pkg is None:
        pkg = types.ModuleType("wfref")
        pkg.__path__ = [ref]
        sys.modules["wfref"] = pkg
        enh = types.ModuleType("wfref.enhancers")
        enh.__path__ = [os.path.join(ref, "enhancers")]
        sys.modules["wfref.enhancers"] = enh
    spec = importlib.util.spec_from_file_location(f"wfref.enhancers.{name}", os.path.join(ref, rel))
    m = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = m
    spec.loader.exec_module(m)
    return m


def hoist_closures(module, fns):
    """Make the @triton.jit helpers a kernel closes over into globals of its module (recursively)."""
    seen = set()
    stack = list(fns)
    while stack:
        f = stack.pop()
        fn = getattr(f, "fn", f)
        if id(fn) in seen:
            continue
        seen.add(id(fn))
        for nm, cell in zip(fn.__code__.co_freevars, fn.__closure__ or ()):
            v = cell.cell_contents
            if hasattr(v, "fn"):
                module.__dict__[nm] = v
                stack.append(v)


# ------------------------------------------------------------------------------------------- inputs
FMT = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
       10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
# byte offsets of the float16 fields of each block format
F16_FIELDS = {2: (0,), 3: (0, 2), 6: (0,), 7: (0, 2), 8: (0,), 10: (80, 82), 11: (108,), 12: (0, 2), 13: (0, 2),
              14: (208,)}


def packed_blocks(rng, qt, n_blocks, special=True):
    """Random packed blocks with finite float16 scales: uniform random bytes everywhere, the float16 fields drawn as
    BASELINE describes (d ~ |N(0,1)| * 0.002 for legacy scales, U(0, 0.01) for K-quant d / dmin); a few blocks get
    edge scales (a subnormal, zero, a large value whose products overflow float16, a negative)."""
    vpb, ts = FMT[qt]
    raw = rng.integers(0, 256, size=(n_blocks, ts), dtype=np.uint8)
    for off in F16_FIELDS[qt]:
        if vpb == 32:
            vals = (np.abs(rng.standard_normal(n_blocks)) * 0.002).astype(np.float16)
            if off == 2:  # the minimum m of Q4_1 / Q5_1 may be negative
                vals = (rng.standard_normal(n_blocks) * 0.01).astype(np.float16)
        else:
            vals = rng.uniform(0, 0.01, n_blocks).astype(np.float16)
        if special and n_blocks >= 8:
            vals[1] = np.float16(3e-7)     # subnormal
            vals[2] = np.float16(0.0)
            vals[3] = np.float16(61000.0)  # products overflow float16
            vals[4] = -vals[4]
        raw[:, off:off + 2] = vals.view(np.uint8).reshape(n_blocks, 2)
    return raw


def make_gguf(ref):
    import triton
    gd = load_ref(ref, "enhancers/gguf_dequant.py", "gguf_dequant")
    gd._get_kernel()
    hoist_closures(gd, [gd._kernel["k"], gd._kernel["add"], gd._kernel["kq"]])
    rng = np.random.default_rng(SEED)
    out = {}
    for qt, (vpb, ts) in FMT.items():
        n_blocks = 32 if vpb == 32 else 4
        raw = packed_blocks(rng, qt, n_blocks)
        out[f"q{qt}_raw"] = raw.reshape(-1)
        n = n_blocks * vpb
        data = torch.from_numpy(raw.reshape(-1).copy())
        for mid in (0, 1, 2):
            for o in (0, 1, 2):
                tdt = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}[o]
                res = torch.empty(n, dtype=tdt)
                if vpb == 32:
                    f = gd._FORMATS[qt]
                    _n, ts_, has_m, qh, qs, sub, is_q8 = f
                    gd._kernel["k"][(triton.cdiv(n_blocks, 32),)](
                        data, res, n_blocks, TS=ts_, HAS_M=has_m, QH=qh, QS=qs, SUB=sub, IS_Q8=is_q8, MID=mid,
                        OUT=o, BB=32)
                else:
                    gd._kernel["kq"][(triton.cdiv(n, 1024),)](data, res, n, FMT=qt, MID=mid, OUT=o, BLOCK=1024)
                bits = res.view(torch.int16).numpy().view(np.uint16) if o != 2 else res.numpy()
                out[f"q{qt}_m{mid}_o{o}"] = bits.copy()
    # LoRA: dequant + first LoRA (DEQ) and a further LoRA (no DEQ), legacy Q8_0 / Q4_1 and K-quant Q4_K
    for qt in (8, 3, 12):
        vpb, ts = FMT[qt]
        n_blocks = 32 if vpb == 32 else 4
        raw = out[f"q{qt}_raw"].reshape(n_blocks, ts)
        n = n_blocks * vpb
        diff = (rng.standard_normal(n) * 0.01).astype(np.float32)
        diff2 = (rng.standard_normal(n) * 0.01).astype(np.float32)
        out[f"lora_q{qt}_diff"], out[f"lora_q{qt}_diff2"] = diff, diff2
        for mid in (0, 1):
            for o in (1, 0):
                tdt = {0: torch.float16, 1: torch.bfloat16}[o]
                res = torch.empty(n, dtype=tdt)
                f = gd._FORMATS[qt] if qt in gd._FORMATS else gd._FORMATS[8]
                _n, ts_, has_m, qh, qs, sub, is_q8 = f
                data = torch.from_numpy(raw.reshape(-1).copy())
                if qt in gd._FORMATS:
                    gd._kernel["add"][(triton.cdiv(n, 1024),)](
                        data, torch.from_numpy(diff), res, n, 0.75, DEQ=True, TS=ts_, HAS_M=has_m, QH=qh, QS=qs,
                        SUB=sub, IS_Q8=is_q8, MID=mid, OUT=o, BLOCK=1024)
                else:  # K-quant: dequantised first, then every LoRA added by the add kernel
                    gd._kernel["kq"][(triton.cdiv(n, 1024),)](data, res, n, FMT=qt, MID=mid, OUT=o, BLOCK=1024)
                    gd._kernel["add"][(triton.cdiv(n, 1024),)](
                        data, torch.from_numpy(diff), res, n, 0.75, DEQ=False, TS=ts_, HAS_M=has_m, QH=qh, QS=qs,
                        SUB=sub, IS_Q8=is_q8, MID=mid, OUT=o, BLOCK=1024)
                gd._kernel["add"][(triton.cdiv(n, 1024),)](
                    data, torch.from_numpy(diff2), res, n, -1.25, DEQ=False, TS=ts_, HAS_M=has_m, QH=qh, QS=qs,
                    SUB=sub, IS_Q8=is_q8, MID=mid, OUT=o, BLOCK=1024)
                out[f"lora_q{qt}_m{mid}_o{o}"] = res.view(torch.int16).numpy().view(np.uint16).copy()
    out["lora_sa"] = np.array([0.75, -1.25], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "gguf_dequant.npz"), **out)
    print("gguf_dequant.npz:", len(out), "arrays")


def _bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def make_fused(ref):
    """The fused-block kernels: _mod, _lnmod, _rms128 (fused_kernels.py), _rope_rows (sage_fused.py) and the int8
    row quantiser _quant_row with each PRE operation (fused_kernels.py:137-174)."""
    import triton
    fk = load_ref(ref, "enhancers/fused_kernels.py", "fused_kernels")
    ks = fk._get_kernels()
    hoist_closures(fk, [ks[k].fn for k in ks])
    sf = load_ref(ref, "enhancers/sage_fused.py", "sage_fused")
    sf._get_kernel()
    g = torch.Generator().manual_seed(SEED + 7)
    out = {}
    # modulate: rows of D = 1024 in 3 groups of 4 rows
    R, D, RPG = 12, 1024, 4
    x = (torch.randn(R, D, generator=g) * 1.5).to(torch.bfloat16)
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-30, 3e38, -3e38, 65504.0, 1.0, -1.0])
    scale = (torch.randn(R // RPG, D, generator=g) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(R // RPG, D, generator=g) * 0.1).to(torch.bfloat16)
    s1 = (1 + scale).contiguous()  # the bf16 (1 + scale) the reference's host code makes
    o = torch.empty_like(x)
    ks["mod"].fn[(R,)](x, s1, shift, o, D, RPG, BLOCK=D)
    out.update(mod_x=_bf16_bits(x), mod_s1=_bf16_bits(s1), mod_shift=_bf16_bits(shift), mod_out=_bf16_bits(o),
               mod_rpg=np.array([RPG]))
    # LayerNorm (no affine, eps 1e-6) + modulate: K = 1024 and 2048
    for K in (1024, 2048):
        xl = (torch.randn(R, K, generator=g) * 2.0 + 0.3).to(torch.bfloat16)
        sc = (torch.randn(R // RPG, K, generator=g) * 0.1).to(torch.bfloat16)
        sh = (torch.randn(R // RPG, K, generator=g) * 0.1).to(torch.bfloat16)
        s1 = (1 + sc).contiguous()
        o = torch.empty_like(xl)
        ks["lnmod"].fn[(R,)](xl, s1, sh, o, RPG, 1e-6, K=K)
        out.update({f"lnmod{K}_x": _bf16_bits(xl), f"lnmod{K}_s1": _bf16_bits(s1), f"lnmod{K}_shift": _bf16_bits(sh),
                    f"lnmod{K}_out": _bf16_bits(o)})
    # RMSNorm over 128 (rs 0: rsqrt.approx), 40 rows (two programs of 32, the second masked)
    n = 40
    xr = (torch.randn(n, 128, generator=g) * 1.2).to(torch.bfloat16)
    w = (1 + torch.randn(128, generator=g) * 0.02).to(torch.bfloat16)
    o = torch.empty_like(xr)
    ks["rms128"].fn[(triton.cdiv(n, 32),)](xr, w, o, n, 1e-6, ROWS=32, RS=0)
    out.update(rms_x=_bf16_bits(xr), rms_w=_bf16_bits(w), rms_out=_bf16_bits(o))
    # RMSNorm-128 + split-half RoPE on (B, L, H, 128) with rotations (1, L, 1, 64, 2, 2) float32
    B, L, H = 2, 6, 4
    xq = (torch.randn(B, L, H, 128, generator=g)).to(torch.bfloat16)
    ang = torch.rand(L, 64, generator=g) * 6.2831853
    f = torch.stack([torch.cos(ang), -torch.sin(ang), torch.sin(ang), torch.cos(ang)], dim=-1)
    f = f.reshape(1, L, 1, 64, 2, 2).float().contiguous()
    wq = (1 + torch.randn(128, generator=g) * 0.02).to(torch.bfloat16)
    o = torch.empty_like(xq)
    n = B * L * H
    sf._kernel["rope_rows"][(triton.cdiv(n, 32),)](xq, f, wq, o, n, H, L, 1e-6, f.stride(1), f.stride(3),
                                                   f.stride(4), f.stride(5), ROWS=32)
    out.update(rope_x=_bf16_bits(xq), rope_f=f.numpy().copy(), rope_w=_bf16_bits(wq), rope_out=_bf16_bits(o),
               rope_shape=np.array([B, L, H]))
    # int8 row quantiser with rotation (ConvRot 256): PRE none / gelu / mod / lnmod, K = 1024, 12 rows
    K = 1024
    xs = (torch.randn(R, K, generator=g) * 1.3).to(torch.bfloat16)
    xs[3] = 0  # an all-zero row: scale 1e-30, int8 0
    sc = (torch.randn(R // RPG, K, generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn(R // RPG, K, generator=g) * 0.1).to(torch.bfloat16)
    s1 = (1 + sc).contiguous()
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    gelu_tab = torch.nn.functional.gelu(allbf).contiguous()
    out.update(q_x=_bf16_bits(xs), q_s1=_bf16_bits(s1), q_shift=_bf16_bits(sh), q_gelu=_bf16_bits(gelu_tab))
    for pre in (0, 1, 2, 3):
        q = torch.empty(R, K, dtype=torch.int8)
        qs = torch.empty(R, 1, dtype=torch.float32)
        if pre == 1:
            ks["quant_row"].fn[(R,)](xs, gelu_tab, xs, q, qs, 1, 0.0, K=K, PRE=1)
        elif pre == 0:
            ks["quant_row"].fn[(R,)](xs, xs, xs, q, qs, 1, 0.0, K=K, PRE=0)
        else:
            ks["quant_row"].fn[(R,)](xs, s1, sh, q, qs, RPG, 1e-6, K=K, PRE=pre)
        out[f"q_pre{pre}_q"] = q.numpy().copy()
        out[f"q_pre{pre}_scale"] = qs.numpy().reshape(-1).copy()
    np.savez_compressed(os.path.join(HERE, "fused_block.npz"), **out)
    print("fused_block.npz:", len(out), "arrays")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the ComfyUI-WeightFerry source folder")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    patch_interpreter()
    if a.only in (None, "gguf"):
        make_gguf(a.ref)
    if a.only in (None, "fused"):
        make_fused(a.ref)


if __name__ == "__main__":
    main()
