"""Python driver of the CPU oracle (oracle.cpp) — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker / the timed CPU restatement of the reference. The
GGUF is parsed here with gguf-py (independently of libda3b's own C++ reader) and
the tensors are handed to the oracle as raw host pointers.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "oracle.cpp")
LIB = os.path.join(HERE, "liboracle.so")
# x86-64-v3 (AVX2/FMA): portable to the GPU hosts; -ffp-contract=off keeps f32
# arithmetic in the written order (no fused multiply-add reassociation).
CXXFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=c++17",
            "-fvisibility=hidden"]


# The DA3cpplib checkout's src/ folder: $DA3_REFERENCE_SRC, else a checkout named
# "reference" beside this repository's root. Where neither exists (a machine without
# the checkout), the prebuilt oracle/_ref library is used as shipped.
REF_SRC_DIR = os.environ.get("DA3_REFERENCE_SRC") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                  "reference", "src")
REF_DIR = os.path.join(HERE, "_ref")
REF_LIB = os.path.join(REF_DIR, "libda3ref.so")
# DA3cpplib's own host-only sources on the path, compiled unmodified (never copied).
REF_SOURCES = ["preprocess.cpp", "uv_posembed.cpp", "nested.cpp", "ray_pose.cpp", "linalg.cpp", "rope2d.cpp",
               "dino_backbone.cpp"]


def build_ref(force: bool = False):
    """Compile the reference's preprocess.cpp, uv_posembed.cpp, nested.cpp, ray_pose.cpp,
    linalg.cpp, rope2d.cpp and dino_backbone.cpp with ref_wrap.cpp and ref_stubs.cpp into
    oracle/_ref/libda3ref.so. Returns the library path, or None when the reference
    checkout is absent (the prebuilt library, if shipped, is still used)."""
    srcs = [os.path.join(REF_SRC_DIR, f) for f in REF_SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return REF_LIB if os.path.exists(REF_LIB) else None
    wrap = os.path.join(HERE, "ref_wrap.cpp")
    stubs = os.path.join(HERE, "ref_stubs.cpp")
    shim = [os.path.join(HERE, "ref_shim", f) for f in os.listdir(os.path.join(HERE, "ref_shim"))]
    newest = max(os.path.getmtime(s) for s in srcs + [wrap, stubs] + shim)
    if force or not os.path.exists(REF_LIB) or os.path.getmtime(REF_LIB) < newest:
        os.makedirs(REF_DIR, exist_ok=True)
        # x86-64 baseline ISA: no FMA, so no contraction; the reference's Release flags
        # (-O3, C++17) otherwise.
        cmd = (["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
                "-I", os.path.join(HERE, "ref_shim"), "-I", REF_SRC_DIR] + srcs + [wrap, stubs, "-o", REF_LIB + ".tmp"])
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference build failed:\n{r.stderr}")
        os.replace(REF_LIB + ".tmp", REF_LIB)
    return REF_LIB


_ref = None


def ref_lib():
    """ctypes handle of oracle/_ref/libda3ref.so, or None when it is unavailable."""
    global _ref
    if _ref is None:
        path = build_ref()
        if path is None:
            return None
        R = ctypes.CDLL(path)
        R.ref_preprocess.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                     ctypes.c_int64, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                     ctypes.c_void_p, ctypes.c_int64]
        R.ref_resize.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p]
        R.ref_uv_pos_embed.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float, ctypes.c_void_p]
        R.ref_ray_pose.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 3
        R.ref_qr.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        R.ref_ql3.argtypes = [ctypes.c_void_p] * 3
        R.ref_smallest_eigvec.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        R.ref_homography.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
        R.ref_rope_tables.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                      ctypes.c_void_p]
        R.ref_interp_pos_embed.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p]
        R.ref_select_saddle.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        R.ref_nested_align.restype = ctypes.c_float
        R.ref_nested_align.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        _ref = R
    return _ref


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["g++"] + CXXFLAGS + [SRC, "-o", LIB + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


class OrTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("type", ctypes.c_int),
                ("ne", ctypes.c_int64 * 4)]


class OrConfig(ctypes.Structure):
    _fields_ = [
        ("patch_size", ctypes.c_int), ("embed_dim", ctypes.c_int), ("depth", ctypes.c_int),
        ("num_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("mlp_hidden", ctypes.c_int),
        ("pos_embed_grid", ctypes.c_int), ("alt_start", ctypes.c_int), ("rope_start", ctypes.c_int),
        ("qknorm_start", ctypes.c_int), ("rope_freq", ctypes.c_float), ("ln_eps", ctypes.c_float),
        ("interp_offset", ctypes.c_float), ("cat_token", ctypes.c_int), ("head_pos_embed", ctypes.c_int),
        ("is_da2", ctypes.c_int), ("head_features", ctypes.c_int), ("n_out_layers", ctypes.c_int),
        ("out_layers", ctypes.c_int * 4), ("head_out_channels", ctypes.c_int * 4),
        ("img_mean", ctypes.c_float * 3), ("img_std", ctypes.c_float * 3), ("resize_target", ctypes.c_int),
        ("resize_upper", ctypes.c_int), ("head_max_depth", ctypes.c_float), ("act_quant", ctypes.c_int),
        ("n_threads", ctypes.c_int),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        L.or_create.restype = ctypes.c_void_p
        L.or_create.argtypes = [ctypes.POINTER(OrConfig), ctypes.POINTER(OrTensor), ctypes.c_int]
        L.or_destroy.argtypes = [ctypes.c_void_p]
        L.or_quantize_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.or_preprocess.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
        L.or_infer.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_infer_mv.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_preprocess_cfg.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
        L.or_resize.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p]
        L.or_uv_pos_embed.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float, ctypes.c_void_p]
        L.or_infer_chw.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_nested_align.restype = ctypes.c_float
        L.or_nested_align.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        L.or_ray_pose.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 3
        L.or_qr.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        L.or_ql3.argtypes = [ctypes.c_void_p] * 3
        L.or_smallest_eigvec.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.or_homography.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
        L.or_set_capture_resid.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_rope_tables.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                     ctypes.c_void_p]
        L.or_interp_pos_embed.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_void_p]
        L.or_select_saddle.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_linear_q8.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.or_get.restype = ctypes.c_int64
        L.or_get.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.POINTER(ctypes.c_float))]
        L.or_dims.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_int)] * 6
        _lib = L
    return _lib


def read_gguf(path):
    """(kv dict, list of (name, ndarray raw, ggml type, ne[4])) via gguf-py."""
    from gguf import GGUFReader

    r = GGUFReader(path)
    kv = {}
    for name, f in r.fields.items():
        if not f.data:
            continue
        tname = f.types[0].name if f.types else ""
        if tname == "STRING":
            kv[name] = bytes(f.parts[f.data[0]]).decode()
        elif tname == "ARRAY":
            vals = [f.parts[i] for i in f.data]
            if f.types[-1].name == "STRING":
                kv[name] = [bytes(v).decode() for v in vals]
            else:
                kv[name] = [v.tolist()[0] for v in vals]
        else:
            kv[name] = f.parts[f.data[0]].tolist()[0]
    tensors = []
    for t in r.tensors:
        ne = [int(v) for v in t.shape] + [1] * (4 - len(t.shape))
        tensors.append((t.name, np.ascontiguousarray(t.data), int(t.tensor_type), ne))
    return kv, tensors


def config_from_kv(kv, act_quant=True, n_threads=0):
    """or_config from GGUF keys; a nested metric-branch file (m_vit.* / m_head.* keys) is
    read the way src/model_loader.cpp:84-127 reads it (head pos-embed off by default)."""
    P = "depthanything3."
    c = OrConfig()
    metric = (P + "m_vit.embed_dim") in kv

    def g(k, d):
        if metric and k.startswith("vit."):
            k = "m_" + k
        elif metric and k.startswith("head.") and k not in ("head.max_depth", "head.has_aux"):
            k = "m_" + k
            if k == "m_head.pos_embed":
                d = False
        return kv.get(P + k, d)
    c.patch_size = g("patch_size", 14)
    c.embed_dim = g("vit.embed_dim", 0)
    c.depth = g("vit.depth", 0)
    c.num_heads = g("vit.num_heads", 0)
    c.head_dim = g("vit.head_dim", 0)
    c.mlp_hidden = g("vit.mlp_hidden", 0)
    c.pos_embed_grid = g("vit.pos_embed_grid", 0)
    c.alt_start = g("vit.alt_start", -1)
    c.rope_start = g("vit.rope_start", -1)
    c.qknorm_start = g("vit.qknorm_start", -1)
    c.rope_freq = g("vit.rope_freq", 100.0)
    c.ln_eps = g("vit.ln_eps", 1e-6)
    c.interp_offset = g("vit.interpolate_offset", 0.1)
    c.cat_token = int(bool(g("vit.cat_token", True)))
    c.head_pos_embed = int(bool(g("head.pos_embed", True)))
    c.is_da2 = int(g("arch", "depthanything3") == "depthanything2")
    c.head_features = g("head.features", 0)
    ol = g("vit.out_layers", [])
    c.n_out_layers = len(ol)
    for i, v in enumerate(ol[:4]):
        c.out_layers[i] = v
    for i, v in enumerate(g("head.out_channels", [])[:4]):
        c.head_out_channels[i] = v
    for i, v in enumerate(g("img.mean", [0.485, 0.456, 0.406])[:3]):
        c.img_mean[i] = v
    for i, v in enumerate(g("img.std", [0.229, 0.224, 0.225])[:3]):
        c.img_std[i] = v
    c.resize_target = g("img.resize_target", 504)
    c.resize_upper = int(not str(g("img.resize_mode", "upper_bound")).startswith("lower"))
    c.head_max_depth = g("head.max_depth", 0.0)
    c.act_quant = int(act_quant)
    c.n_threads = int(n_threads)
    return c


class Oracle:
    """CPU restatement of the reference depth path over a GGUF file."""

    def __init__(self, gguf_path, act_quant=True, n_threads=0, swap=None):
        """swap: optional {name_a: name_b} pairs whose tensors trade places (tests that
        route one head's weights through another head's code)."""
        L = lib()
        self.kv, self._tensors = read_gguf(gguf_path)
        if swap:
            pairs = dict(swap)
            pairs.update({b: a for a, b in swap.items()})
            self._tensors = [(pairs.get(n, n), d, t, ne) for n, d, t, ne in self._tensors]
        # metric-branch tensors are also reachable as vit.* / head.* (src/model_loader.cpp:146-154)
        self._tensors = self._tensors + [(n[2:], d, t, ne) for n, d, t, ne in self._tensors
                                         if n.startswith(("m_vit.", "m_head."))]
        self.cfg = config_from_kv(self.kv, act_quant, n_threads)
        arr = (OrTensor * len(self._tensors))()
        self._names = []
        for i, (name, data, typ, ne) in enumerate(self._tensors):
            nb = name.encode()
            self._names.append(nb)
            arr[i].name = nb
            arr[i].data = data.ctypes.data
            arr[i].type = typ
            for k in range(4):
                arr[i].ne[k] = ne[k]
        self._arr = arr
        self.h = L.or_create(ctypes.byref(self.cfg), arr, len(self._tensors))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_destroy(self.h)
            self.h = None

    def tensor(self, name):
        for n, d, t, ne in self._tensors:
            if n == name:
                return d, t, ne
        return None

    def get(self, name):
        p = ctypes.POINTER(ctypes.c_float)()
        n = lib().or_get(self.h, name.encode(), ctypes.byref(p))
        if n < 0:
            return None
        if n == 0:
            return np.zeros(0, dtype=np.float32)
        return np.ctypeslib.as_array(p, shape=(n,)).copy()

    def set_capture_residuals(self, on=True):
        """Keep the residual stream after every ViT block of later forwards ("x<i>")."""
        lib().or_set_capture_resid(self.h, int(on))

    def residual(self, layer):
        """Residual stream after block `layer` of the last forward, [rows][embed_dim]."""
        v = self.get(f"x{layer}")
        return None if v is None else v.reshape(-1, self.cfg.embed_dim)

    def dims(self):
        v = [ctypes.c_int() for _ in range(6)]
        lib().or_dims(self.h, *[ctypes.byref(x) for x in v])
        return tuple(x.value for x in v)

    def preprocess(self, rgb, legacy=False):
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w = rgb.shape[:2]
        H, W = ctypes.c_int(), ctypes.c_int()
        buf = np.zeros(3 * (h + 64) * (w + 64) * 4, dtype=np.float32)
        rc = lib().or_preprocess(self.h, rgb.ctypes.data, w, h, int(legacy), buf.ctypes.data, ctypes.byref(H),
                                 ctypes.byref(W))
        assert rc == 0
        return buf[: 3 * H.value * W.value].reshape(3, H.value, W.value).copy()

    def infer(self, rgb, legacy=False, aux=False):
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w = rgb.shape[:2]
        rc = lib().or_infer(self.h, rgb.ctypes.data, w, h, int(legacy), int(aux))
        if rc != 0:
            raise RuntimeError(f"oracle infer failed {rc}")
        return self._outputs(aux)

    def _outputs(self, aux):
        H, W, od, ah, aw, _ = self.dims()
        out = {"H": H, "W": W, "depth": self.get("depth").reshape(H, W), "logits": self.get("logits").reshape(od, H, W)}
        conf = self.get("conf")
        if conf is not None and conf.size:
            out["conf"] = conf.reshape(H, W)
        if aux and ah > 0:
            out["aux"] = self.get("aux").reshape(7, ah, aw)
        pose = self.get("pose")
        if pose is not None and pose.size:  # [9 pose encoding | 12 extrinsics | 9 intrinsics]
            out["pose"] = pose.reshape(30)
        sky = self.get("sky")
        if sky is not None and sky.size:
            out["sky"] = sky.reshape(H, W)
        return out

    def infer_chw(self, chw, aux=False):
        """Forward from a normalised planar f32 image [3][H][W] (no preprocessing)."""
        chw = np.ascontiguousarray(chw, dtype=np.float32)
        _, H, W = chw.shape
        rc = lib().or_infer_chw(self.h, chw.ctypes.data, H, W, int(aux))
        if rc != 0:
            raise RuntimeError(f"oracle infer_chw failed {rc}")
        return self._outputs(aux)

    def infer_mv(self, rgbs, legacy=True, aux=False):
        rgbs = [np.ascontiguousarray(r, dtype=np.uint8) for r in rgbs]
        S = len(rgbs)
        h, w = rgbs[0].shape[:2]
        ptrs = (ctypes.c_void_p * S)(*[r.ctypes.data for r in rgbs])
        rc = lib().or_infer_mv(self.h, ptrs, S, w, h, int(legacy), int(aux))
        if rc != 0:
            raise RuntimeError(f"oracle infer_mv failed {rc}")
        H, W, od, ah, aw, b_idx = self.dims()
        out = {"H": H, "W": W, "b_idx": b_idx, "depth": self.get("depth").reshape(S, H, W),
               "conf": self.get("conf").reshape(S, H, W), "logits": self.get("logits").reshape(S, od, H, W)}
        if aux and ah > 0:
            out["aux"] = self.get("aux").reshape(S, 7, ah, aw)
        pose = self.get("pose")
        if pose is not None and pose.size:
            out["pose"] = pose.reshape(S, 30)
        return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.zeros(x.size // 32 * 34, dtype=np.uint8)
    lib().or_quantize_q8_0(x.ctypes.data, x.size, out.ctypes.data)
    return out


# ---------------------------------------------------------------- preprocessing pins
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _policy_args(mean, std):
    m = np.ascontiguousarray(mean, dtype=np.float32)
    s = np.ascontiguousarray(std, dtype=np.float32)
    return m, s


def preprocess_cfg(rgb, patch=14, target=504, upper=True, legacy=False, mean=IMAGENET_MEAN, std=IMAGENET_STD,
                   impl="oracle"):
    """preprocess_real / legacy preprocess with an explicit policy -> CHW f32.
    impl="oracle" runs the restatement, impl="ref" the reference's own preprocess.cpp."""
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w = rgb.shape[:2]
    m, s = _policy_args(mean, std)
    big = int(max(h, w) * max(1.0, target / min(h, w))) + 2 * patch + 2
    cap = 3 * big * big
    out = np.zeros(cap, dtype=np.float32)
    H, W = ctypes.c_int(), ctypes.c_int()
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        rc = R.ref_preprocess(rgb.ctypes.data, w, h, patch, target, int(upper), m.ctypes.data, s.ctypes.data,
                              int(legacy), out.ctypes.data, cap, ctypes.byref(H), ctypes.byref(W), None, 0)
    else:
        rc = lib().or_preprocess_cfg(rgb.ctypes.data, w, h, patch, target, int(upper), m.ctypes.data, s.ctypes.data,
                                     int(legacy), out.ctypes.data, cap, ctypes.byref(H), ctypes.byref(W))
    if rc != 0:
        raise RuntimeError(f"preprocess failed ({impl}): {rc}")
    return out[: 3 * H.value * W.value].reshape(3, H.value, W.value).copy()


def resize_u8(rgb, dw, dh, mode, impl="oracle"):
    """uint8 HWC resize: mode "cubic" or "area"."""
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w = rgb.shape[:2]
    out = np.zeros((dh, dw, 3), dtype=np.uint8)
    md = {"cubic": 0, "area": 1}[mode]
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        rc = R.ref_resize(rgb.ctypes.data, w, h, dw, dh, md, out.ctypes.data)
    else:
        rc = lib().or_resize(rgb.ctypes.data, w, h, dw, dh, md, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"resize failed ({impl}): {rc}")
    return out


def uv_pos_embed(pw, ph, C, aspect, impl="oracle"):
    """Raw UV embedding, [ph][pw][C]."""
    out = np.zeros((ph, pw, C), dtype=np.float32)
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        rc = R.ref_uv_pos_embed(pw, ph, C, aspect, out.ctypes.data)
    else:
        rc = lib().or_uv_pos_embed(pw, ph, C, aspect, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"uv_pos_embed failed ({impl}): {rc}")
    return out


def nested_align(any_depth, any_conf, any_ext, any_intr, metric_depth, sky, impl="oracle"):
    """Nested metric alignment (src/nested.cpp:22-96: sky fill of the metric depth, then
    the alignment). impl="oracle" runs the restatement, impl="ref" the reference's own
    nested.cpp. Returns (depth, ext [12], scale)."""
    a = [np.ascontiguousarray(x, dtype=np.float32).reshape(-1) for x in
         (any_depth, any_conf, any_ext, any_intr, metric_depth, sky)]
    a[4] = a[4].copy()
    n = a[0].size
    out = np.zeros(n, np.float32)
    ext = np.zeros(12, np.float32)
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        fn = R.ref_nested_align
    else:
        fn = lib().or_nested_align
    scale = fn(*[x.ctypes.data for x in a], n, out.ctypes.data, ext.ctypes.data)
    return out, ext, float(scale)


def _impl(impl, name):
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        return getattr(R, "ref_" + name)
    return getattr(lib(), "or_" + name)


def ray_pose(ray, conf, img_h, img_w, impl="oracle"):
    """Ray->pose solver (src/ray_pose.cpp:95-252, production defaults) on an interleaved
    ray field [Hy][Wx][6] and confidence [Hy][Wx]. Returns (ext [3][4] camera-to-world,
    intr [3][3], diag dict) or None when the solver reports a degenerate field."""
    ray = np.ascontiguousarray(ray, dtype=np.float32)
    conf = np.ascontiguousarray(conf, dtype=np.float32)
    Hy, Wx = conf.shape
    ext = np.zeros(12, np.float32)
    intr = np.zeros(9, np.float32)
    diag = np.zeros(26, np.float64)
    rc = _impl(impl, "ray_pose")(ray.ctypes.data, conf.ctypes.data, Hy, Wx, img_h, img_w, ext.ctypes.data,
                                 intr.ctypes.data, diag.ctypes.data)
    if rc != 0:
        return None
    d = {"R": diag[:9].reshape(3, 3), "T": diag[9:12], "focal": diag[12:14], "pp": diag[14:16],
         "A": diag[16:25].reshape(3, 3), "n_inlier_best": int(diag[25])}
    return ext.reshape(3, 4), intr.reshape(3, 3), d


def qr(a, impl="oracle"):
    a = np.ascontiguousarray(a, dtype=np.float64)
    n = a.shape[0]
    q = np.zeros((n, n)); r = np.zeros((n, n))
    _impl(impl, "qr")(a.ctypes.data, n, q.ctypes.data, r.ctypes.data)
    return q, r


def ql3(a, impl="oracle"):
    a = np.ascontiguousarray(a, dtype=np.float64)
    q = np.zeros((3, 3)); l = np.zeros((3, 3))
    _impl(impl, "ql3")(a.ctypes.data, q.ctypes.data, l.ctypes.data)
    return q, l


def smallest_eigvec(m, impl="oracle"):
    m = np.ascontiguousarray(m, dtype=np.float64)
    v = np.zeros(m.shape[0])
    _impl(impl, "smallest_eigvec")(m.ctypes.data, m.shape[0], v.ctypes.data)
    return v


def homography(src, dst, w, impl="oracle"):
    src = np.ascontiguousarray(src, dtype=np.float64)
    dst = np.ascontiguousarray(dst, dtype=np.float64)
    w = np.ascontiguousarray(w, dtype=np.float64)
    H = np.zeros(9)
    rc = _impl(impl, "homography")(src.ctypes.data, dst.ctypes.data, w.ctypes.data, w.size, H.ctypes.data)
    return H.reshape(3, 3) if rc == 0 else None


# ---------------------------------------------------------------- DA3 host-code pins
def _impl_lib(impl):
    if impl == "ref":
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        return R, "ref_"
    return lib(), "or_"


def rope_tables(pos_yx, head_dim=64, freq=100.0, impl="oracle"):
    """2-D RoPE cos / sin tables [tokens][head_dim] for positions pos_yx [tokens][2]."""
    L, pre = _impl_lib(impl)
    pos = np.ascontiguousarray(pos_yx, dtype=np.float32)
    T = pos.shape[0]
    c = np.zeros((T, head_dim), np.float32)
    s = np.zeros((T, head_dim), np.float32)
    rc = getattr(L, pre + "rope_tables")(pos.ctypes.data, T, head_dim, float(freq), c.ctypes.data, s.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"rope_tables failed ({impl})")
    return c, s


def interp_pos_embed(pos_embed, grid, gh, gw, offset=0.1, impl="oracle"):
    """Offset bicubic interpolation of a pos-embed table [1 + grid^2][embed] to gh x gw."""
    L, pre = _impl_lib(impl)
    pe = np.ascontiguousarray(pos_embed, dtype=np.float32)
    E = pe.shape[1]
    out = np.zeros((1 + gh * gw, E), np.float32)
    rc = getattr(L, pre + "interp_pos_embed")(pe.ctypes.data, E, grid, float(offset), gh, gw, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"interp_pos_embed failed ({impl})")
    return out


def select_saddle(cls, impl="oracle"):
    """Index of the reference view chosen from S CLS vectors [S][embed]."""
    L, pre = _impl_lib(impl)
    c = np.ascontiguousarray(cls, dtype=np.float32)
    return int(getattr(L, pre + "select_saddle")(c.ctypes.data, c.shape[0], c.shape[1]))


def linear_q8(x, wq8, N, bias=None, act_quant=True):
    """linear() of x f32 [M][K] with a Q8_0 weight (GGUF bytes [N][K/32][34]); act_quant
    follows ggml's Q8_0 x Q8_0 CPU dot product. Returns y f32 [M][N]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    w = np.ascontiguousarray(wq8, dtype=np.uint8)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros((M, N), np.float32)
    lib().or_linear_q8(x.ctypes.data, M, K, w.ctypes.data, N, b.ctypes.data if b is not None else None,
                       int(act_quant), y.ctypes.data)
    return y
