"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the DA3cpplib checkout (for oracle/_ref), gguf-py and
transformers:  python tests/golden/make_golden.py

Fixtures (all small):
  preprocess_ref.npz   DA3cpplib's own src/preprocess.cpp and src/uv_posembed.cpp,
                       compiled unmodified into oracle/_ref, on seeded uint8 images:
                       preprocess_real (upper/lower bound, cubic and area paths,
                       patch rounding), the legacy floor-to-patch path, the two uint8
                       resizers, and the UV embedding.
  q8_0_ggufpy.npz      gguf-py's Q8_0 quantiser (quants.py, bit-exact with ggml's C
                       reference quantiser) on seeded f32 rows, ties included.
  da2_hf_tiny.gguf     A random DA2 model (DINOv2 backbone + DPT head) built with
  da2_hf_tiny.npz      transformers' DepthAnythingForDepthEstimation, converted to
                       DA3cpplib's GGUF layout (ViT linears Q8_0, the model's linear
                       weights replaced by their Q8_0 round trip; everything else f32),
                       with transformers' f32
                       outputs (pre-activation logits, relative depth, the four
                       normalised backbone features) for a square image at the
                       position-embedding grid and a non-square one. transformers'
                       position-embedding interpolation is replaced by DINOv2's
                       published offset rule (bicubic, scale (g + 0.1) / grid, applied
                       at every grid), which is the rule src/dino_backbone.cpp:18-56
                       follows.
  linalg_ref.json      The known answers of DA3cpplib's own tests/test_linalg.cpp (its
                       fixed 3x3 matrix with torch.linalg.qr and the torch-derived QL
                       factors, the 4x4 symmetric eigen case, the 12-point homography
                       recovery), parsed from that file.
  raypose_ref.npz      DA3cpplib's own src/ray_pose.cpp + src/linalg.cpp, compiled
                       unmodified into oracle/_ref, on the seeded synthetic ray fields
                       of tests/rayfield.py: extrinsics, intrinsics and the solver's
                       double diagnostics.
  nested_ref.npz       DA3cpplib's own src/nested.cpp (oracle/_ref) on seeded inputs:
                       aligned depth, extrinsics and scale.
  da3_host_ref.npz     DA3cpplib's own src/rope2d.cpp and src/dino_backbone.cpp host
                       functions (oracle/_ref): build_rope_tables on the backbone's
                       local and global ("no-diff") position grids and on random
                       positions, DinoBackbone::interp_pos_embed (offset bicubic) from
                       the 37-grid to the C1-C4 grids and odd grids, and
                       select_reference_view_saddle on seeded CLS sets of 3-8 views.
                       Small cases store the full outputs; the full-size C3/C4 tables
                       store a SHA-256 of their bytes (da3_host_cases()).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as orc  # noqa: E402

SEED = 20261201

# (h, w, patch, target, upper, legacy) — each exercises a different branch of
# preprocess_real: cubic upscale, area downscale, lower bound, patch-rounding resize,
# no-op, and the legacy bilinear floor path.
PRE_CASES = [
    (37, 53, 14, 56, 1, 0),
    (90, 61, 14, 56, 1, 0),
    (37, 53, 14, 42, 0, 0),
    (56, 70, 14, 70, 1, 0),
    (49, 49, 14, 56, 0, 0),
    (29, 45, 14, 28, 1, 0),
    (40, 33, 14, 504, 1, 1),
    (15, 100, 14, 84, 1, 0),
]
RESIZE_CASES = [(23, 31, 57, 40, "cubic"), (23, 31, 12, 9, "area"), (40, 40, 17, 13, "area"), (11, 7, 30, 19, "cubic"),
                (64, 48, 21, 48, "area")]
UV_CASES = [(8, 8, 32, 1.0), (5, 4, 16, 5 / 4), (13, 19, 64, 13 / 19)]


def make_preprocess():
    if orc.ref_lib() is None:
        raise SystemExit("oracle/_ref could not be built: the DA3cpplib checkout is required")
    rng = np.random.default_rng(SEED)
    out = {}
    for i, (h, w, patch, target, upper, legacy) in enumerate(PRE_CASES):
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        out[f"pre{i}_in"] = img
        out[f"pre{i}_cfg"] = np.array([patch, target, upper, legacy], dtype=np.int32)
        out[f"pre{i}_out"] = orc.preprocess_cfg(img, patch, target, bool(upper), bool(legacy), impl="ref")
    for i, (h, w, dw, dh, mode) in enumerate(RESIZE_CASES):
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        out[f"rs{i}_in"] = img
        out[f"rs{i}_cfg"] = np.array([dw, dh, 0 if mode == "cubic" else 1], dtype=np.int32)
        out[f"rs{i}_out"] = orc.resize_u8(img, dw, dh, mode, impl="ref")
    for i, (pw, ph, C, aspect) in enumerate(UV_CASES):
        out[f"uv{i}_cfg"] = np.array([pw, ph, C, aspect], dtype=np.float64)
        out[f"uv{i}_out"] = orc.uv_pos_embed(pw, ph, C, aspect, impl="ref")
    np.savez_compressed(os.path.join(HERE, "preprocess_ref.npz"), **out)


def make_q8():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    rng = np.random.default_rng(SEED + 1)
    x = rng.standard_normal((64, 256), dtype=np.float32) * rng.uniform(0.01, 10, size=(64, 1)).astype(np.float32)
    # rows with exact ties (x * 127 / amax lands on k + 0.5) and zero blocks
    t = np.tile(np.arange(-16, 16, dtype=np.float32) + 0.5, 8)
    t[0] = 127.0
    x[0] = t * (1.0 / 127.0)
    x[1, :32] = 0.0
    x[2, :] = np.float32(1e-30)
    q = quants.quantize(x, GGMLQuantizationType.Q8_0)
    np.savez_compressed(os.path.join(HERE, "q8_0_ggufpy.npz"), x=x, q=np.ascontiguousarray(q).reshape(-1))


# ----------------------------------------------------------------------- DA2 via HF
HF_D, HF_HEADS, HF_LAYERS, HF_GRID = 128, 2, 4, 4
HF_OC, HF_F = (16, 32, 64, 64), 32


def _hf_model():
    import torch
    from transformers import DepthAnythingConfig, DepthAnythingForDepthEstimation, Dinov2Config

    bb = Dinov2Config(hidden_size=HF_D, num_hidden_layers=HF_LAYERS, num_attention_heads=HF_HEADS, mlp_ratio=2,
                      image_size=14 * HF_GRID, patch_size=14, layerscale_value=1.0, hidden_act="gelu",
                      layer_norm_eps=1e-6, qkv_bias=True, out_features=[f"stage{i}" for i in range(1, HF_LAYERS + 1)],
                      apply_layernorm=True, reshape_hidden_states=False)
    cfg = DepthAnythingConfig(backbone_config=bb, reassemble_hidden_size=HF_D, neck_hidden_sizes=list(HF_OC),
                              fusion_hidden_size=HF_F, head_hidden_size=32, depth_estimation_type="relative",
                              patch_size=14)
    torch.manual_seed(SEED + 2)
    m = DepthAnythingForDepthEstimation(cfg).eval()
    g = torch.Generator().manual_seed(SEED + 3)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "mask_token" in name:
                continue
            if p.dim() >= 2 and "embeddings" not in name:
                fan_in = p[0].numel() if "resize" not in name or p.shape[-1] == 3 else p.shape[0]
                p.copy_(torch.randn(p.shape, generator=g) / np.sqrt(fan_in))
            elif "norm" in name and name.endswith("weight") or "lambda1" in name:
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(0.1 * torch.randn(p.shape, generator=g))
        # ViT linear weights are stored as Q8_0 in the GGUF: give the model exactly the
        # values the file will hold
        for name, p in m.named_parameters():
            if _is_vit_linear(name):
                p.copy_(torch.from_numpy(_q8_round_trip(p.detach().numpy())))
    return m


def _is_vit_linear(name):
    return "backbone.encoder.layer." in name and name.endswith(".weight") and any(
        k in name for k in ("query.", "key.", "value.", "output.dense.", "fc1.", "fc2."))


def _q8(w):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    return quants.quantize(np.ascontiguousarray(w, dtype=np.float32), GGMLQuantizationType.Q8_0)


def _q8_round_trip(w):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    return quants.dequantize(_q8(w), GGMLQuantizationType.Q8_0).reshape(w.shape).astype(np.float32)


def _hf_to_gguf(m, path, offset):
    """Write the transformers model in DA3cpplib's tensor names / ggml shapes (f32)."""
    import gguf

    sd = {k: v.detach().float().numpy() for k, v in m.state_dict().items()}
    T = []
    add = lambda n, a: T.append((n, np.ascontiguousarray(a, dtype=np.float32), False))
    addq = lambda n, a: T.append((n, _q8(a), True))
    e = "backbone.embeddings."
    add("vit.patch_embed.weight", sd[e + "patch_embeddings.projection.weight"])
    add("vit.patch_embed.bias", sd[e + "patch_embeddings.projection.bias"])
    add("vit.cls_token", sd[e + "cls_token"])
    add("vit.pos_embed", sd[e + "position_embeddings"])
    add("vit.norm.weight", sd["backbone.layernorm.weight"])
    add("vit.norm.bias", sd["backbone.layernorm.bias"])
    for i in range(HF_LAYERS):
        s, p = f"backbone.encoder.layer.{i}.", f"vit.blk.{i}."
        a = s + "attention.attention."
        add(p + "norm1.weight", sd[s + "norm1.weight"])
        add(p + "norm1.bias", sd[s + "norm1.bias"])
        addq(p + "attn_qkv.weight", np.concatenate([sd[a + k + ".weight"] for k in ("query", "key", "value")], 0))
        add(p + "attn_qkv.bias", np.concatenate([sd[a + k + ".bias"] for k in ("query", "key", "value")], 0))
        addq(p + "attn_proj.weight", sd[s + "attention.output.dense.weight"])
        add(p + "attn_proj.bias", sd[s + "attention.output.dense.bias"])
        add(p + "ls1", sd[s + "layer_scale1.lambda1"])
        add(p + "norm2.weight", sd[s + "norm2.weight"])
        add(p + "norm2.bias", sd[s + "norm2.bias"])
        addq(p + "mlp_fc1.weight", sd[s + "mlp.fc1.weight"])
        add(p + "mlp_fc1.bias", sd[s + "mlp.fc1.bias"])
        addq(p + "mlp_fc2.weight", sd[s + "mlp.fc2.weight"])
        add(p + "mlp_fc2.bias", sd[s + "mlp.fc2.bias"])
        add(p + "ls2", sd[s + "layer_scale2.lambda1"])
    r = "neck.reassemble_stage.layers."
    for s in range(4):
        add(f"head.proj.{s}.weight", sd[f"{r}{s}.projection.weight"])
        add(f"head.proj.{s}.bias", sd[f"{r}{s}.projection.bias"])
    for s in (0, 1, 3):
        add(f"head.resize.{s}.weight", sd[f"{r}{s}.resize.weight"])
        add(f"head.resize.{s}.bias", sd[f"{r}{s}.resize.bias"])
    for s in range(4):
        add(f"head.scratch.layer{s + 1}_rn.weight", sd[f"neck.convs.{s}.weight"])
    # transformers' fusion layer k processes the (k+1)-th deepest level: refinenet 4-k
    for k in range(4):
        f, p = f"neck.fusion_stage.layers.{k}.", f"head.scratch.rn{4 - k}."
        units = (("residual_layer2", "rc2"),) if k == 0 else (("residual_layer1", "rc1"), ("residual_layer2", "rc2"))
        for hu, u in units:
            for hc, c in (("convolution1", "c1"), ("convolution2", "c2")):
                add(p + f"{u}.{c}.weight", sd[f + f"{hu}.{hc}.weight"])
                add(p + f"{u}.{c}.bias", sd[f + f"{hu}.{hc}.bias"])
        add(p + "out.weight", sd[f + "projection.weight"])
        add(p + "out.bias", sd[f + "projection.bias"])
    for hc, c in (("conv1", "out1"), ("conv2", "out2a"), ("conv3", "out2b")):
        add(f"head.scratch.{c}.weight", sd[f"head.{hc}.weight"])
        add(f"head.scratch.{c}.bias", sd[f"head.{hc}.bias"])

    w = gguf.GGUFWriter(path + ".tmp", arch="depthanything3")
    P = "depthanything3."
    w.add_string(P + "arch", "depthanything2")
    w.add_string(P + "checkpoint_name", "da2-hf-tiny-random")
    w.add_uint32(P + "patch_size", 14)
    w.add_uint32(P + "vit.embed_dim", HF_D)
    w.add_uint32(P + "vit.depth", HF_LAYERS)
    w.add_uint32(P + "vit.num_heads", HF_HEADS)
    w.add_uint32(P + "vit.head_dim", HF_D // HF_HEADS)
    w.add_uint32(P + "vit.mlp_hidden", 2 * HF_D)
    w.add_string(P + "vit.ffn_type", "mlp")
    w.add_uint32(P + "vit.num_register_tokens", 0)
    for k in ("alt_start", "rope_start", "qknorm_start"):
        w.add_int32(P + "vit." + k, -1)
    w.add_float32(P + "vit.rope_freq", 100.0)
    w.add_bool(P + "vit.cat_token", False)
    w.add_bool(P + "vit.qkv_bias", True)
    w.add_float32(P + "vit.ln_eps", 1e-6)
    w.add_float32(P + "vit.interpolate_offset", float(offset))
    w.add_bool(P + "vit.interpolate_antialias", False)
    w.add_uint32(P + "vit.pos_embed_grid", HF_GRID)
    w.add_array(P + "vit.out_layers", list(range(HF_LAYERS)))
    w.add_array(P + "img.mean", [0.485, 0.456, 0.406])
    w.add_array(P + "img.std", [0.229, 0.224, 0.225])
    w.add_string(P + "img.resize_mode", "lower_bound")
    w.add_uint32(P + "img.resize_target", 14 * HF_GRID)
    w.add_uint32(P + "head.features", HF_F)
    w.add_array(P + "head.out_channels", list(HF_OC))
    w.add_uint32(P + "head.output_dim", 1)
    w.add_bool(P + "head.pos_embed", False)
    w.add_float32(P + "head.max_depth", 0.0)
    w.add_bool(P + "head.has_aux", False)
    from gguf.constants import GGMLQuantizationType

    for n, a, q in T:
        if q:
            w.add_tensor(n, a, raw_dtype=GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(n, a)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(path + ".tmp", path)


def _dinov2_offset_interp(self, embeddings, height, width):
    """DINOv2's published position-embedding interpolation (facebookresearch/dinov2
    vision_transformer.py interpolate_pos_encoding): bicubic with scale_factor
    ((g + 0.1) / grid) per axis, align_corners False."""
    import torch

    pos = self.position_embeddings
    M = int(round((pos.shape[1] - 1) ** 0.5))
    gh, gw = height // self.patch_size, width // self.patch_size
    pp = pos[:, 1:].reshape(1, M, M, -1).permute(0, 3, 1, 2)
    pp = torch.nn.functional.interpolate(pp, scale_factor=((gh + 0.1) / M, (gw + 0.1) / M), mode="bicubic",
                                         align_corners=False)
    assert pp.shape[-2:] == (gh, gw)
    return torch.cat([pos[:, :1], pp.permute(0, 2, 3, 1).reshape(1, gh * gw, -1)], 1)


def make_hf():
    import torch

    m = _hf_model()
    out = {}
    rng = np.random.default_rng(SEED + 4)
    cases = [("sq", 14 * HF_GRID, 14 * HF_GRID), ("rect", 14 * (HF_GRID + 1), 14 * (HF_GRID - 1))]
    for tag, w, h in cases:
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        # the image is already a multiple of 14 with its short side at the target for
        # "sq"; for "rect" legacy=floor-to-patch leaves it unchanged, so the network
        # input is the plain normalisation of the image either way
        chw = orc.preprocess_cfg(img, 14, 14 * HF_GRID, False, legacy=True)
        x = torch.from_numpy(chw)[None]
        cap = {}
        hk = m.head.conv3.register_forward_hook(lambda mod, i, o: cap.__setitem__("logits", o))
        emb = m.backbone.embeddings
        orig = type(emb).interpolate_pos_encoding
        type(emb).interpolate_pos_encoding = _dinov2_offset_interp
        try:
            with torch.no_grad():
                feats = m.backbone(x).feature_maps
                res = m(x)
        finally:
            type(emb).interpolate_pos_encoding = orig
            hk.remove()
        out[f"{tag}_img"] = img
        out[f"{tag}_depth"] = res.predicted_depth[0].numpy()
        out[f"{tag}_logits"] = cap["logits"][0, 0].numpy()
        for i, f in enumerate(feats):
            out[f"{tag}_feat{i}"] = f[0, 1:].numpy()  # normalised, CLS dropped: [Npatch][D]
    _hf_to_gguf(m, os.path.join(HERE, "da2_hf_tiny.gguf"), 0.1)
    np.savez_compressed(os.path.join(HERE, "da2_hf_tiny.npz"), **out)


REF_TESTS = os.path.join(os.path.dirname(orc.REF_SRC_DIR), "tests")
RAY_CASES = [(1, 48, 64, 0.2), (2, 64, 64, 0.5), (3, 40, 56, 0.0), (4, 96, 72, 0.3)]


def make_linalg():
    import json
    import re

    src = open(os.path.join(REF_TESTS, "test_linalg.cpp")).read()

    def arr(name):
        m = re.search(r"\b" + name + r"\s*\[[^\]]*\](?:\[[^\]]*\])?\s*=\s*\{(.*?)\};", src, re.S)
        return [float(v) for v in re.findall(r"-?\d+\.?\d*(?:e-?\d+)?", m.group(1))]

    det = re.search(r"close\(det3\(A\),\s*([-\d.]+)", src).group(1)
    out = {"source": "DA3cpplib tests/test_linalg.cpp", "A": arr("A"), "det": float(det), "QR_Q": arr("QR_Q"),
           "QR_R": arr("QR_R"), "QL_Q": arr("QL_Q"), "QL_L": arr("QL_L"), "M4": arr("M"), "Htrue": arr("Htrue"),
           "pts": arr("pts")}
    assert len(out["A"]) == 9 and len(out["QL_L"]) == 9 and len(out["M4"]) == 16 and len(out["pts"]) == 24
    with open(os.path.join(HERE, "linalg_ref.json"), "w") as f:
        json.dump(out, f, indent=1)


def make_raypose():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import rayfield

    out = {}
    for seed, hy, wx, outl in RAY_CASES:
        ray, conf, _ = rayfield.field(seed, hy, wx, outliers=outl)
        ext, intr, d = orc.ray_pose(ray, conf, hy * 14 // 8, wx * 14 // 8, impl="ref")
        out[f"s{seed}_ext"] = ext
        out[f"s{seed}_intr"] = intr
        out[f"s{seed}_diag"] = np.concatenate([d["R"].ravel(), d["T"], d["focal"], d["pp"], d["A"].ravel(),
                                               [d["n_inlier_best"]]])
    np.savez_compressed(os.path.join(HERE, "raypose_ref.npz"), **out)


NESTED_CASES = [(21, 4096, 0.3), (22, 3000, 0.004), (23, 2500, 0.6)]


def nested_inputs(seed, n, sky_frac):
    rng = np.random.default_rng(seed)
    ad = rng.uniform(0.0, 5.0, n).astype(np.float32)
    ac = rng.uniform(1.0, 3.0, n).astype(np.float32)
    ext = rng.standard_normal(12).astype(np.float32)
    intr = np.array([rng.uniform(100, 400), 0, 56, 0, rng.uniform(100, 400), 56, 0, 0, 1], np.float32)
    md = rng.uniform(0.0, 10.0, n).astype(np.float32)
    sky = np.where(rng.random(n) < sky_frac, rng.uniform(0.3, 1.0, n), rng.uniform(0.0, 0.3, n)).astype(np.float32)
    return ad, ac, ext, intr, md, sky


def make_nested():
    out = {}
    for seed, n, frac in NESTED_CASES:
        d, e, s = orc.nested_align(*nested_inputs(seed, n, frac), impl="ref")
        out[f"s{seed}_depth"] = d
        out[f"s{seed}_ext"] = e
        out[f"s{seed}_scale"] = np.float32(s)
    np.savez_compressed(os.path.join(HERE, "nested_ref.npz"), **out)


def backbone_positions(gh, gw, nodiff=False):
    """Token positions (y, x) of the backbone's RoPE (src/dino_backbone.cpp:242-248):
    token 0 at (0, 0); patch t at (row + 1, col + 1), or (1, 1) for the global layers'
    position-free tables."""
    pos = np.zeros((1 + gh * gw, 2), np.float32)
    for t in range(gh * gw):
        pos[1 + t] = (1, 1) if nodiff else (t // gw + 1, t % gw + 1)
    return pos


def da3_host_cases():
    """(rope cases, interp cases, saddle cases) of da3_host_ref.npz, all seeded.
    rope: (name, positions, head_dim, freq, full) ; interp: (name, pos_embed, grid, gh,
    gw, offset, full) ; saddle: (name, cls [S][E])."""
    rng = np.random.default_rng(SEED + 7)
    rope = [("rl8x9", backbone_positions(8, 9), 64, 100.0, True),
            ("rn8x9", backbone_positions(8, 9, nodiff=True), 64, 100.0, True),
            ("rrand", rng.uniform(0, 60, size=(97, 2)).astype(np.float32), 64, 100.0, True),
            ("rhd32", backbone_positions(5, 3), 32, 10.0, True),
            ("rl36", backbone_positions(36, 36), 64, 100.0, False),
            ("rl37", backbone_positions(37, 37), 64, 100.0, False)]
    interp = []
    for name, grid, gh, gw, E, full in (("p37to36", 37, 36, 36, 8, True), ("p37to37", 37, 37, 37, 8, True),
                                        ("p8to5x7", 8, 5, 7, 16, True), ("p37to36w", 37, 36, 36, 1024, False),
                                        ("p37to37w", 37, 37, 37, 1024, False), ("p4to9x2", 4, 9, 2, 4, True)):
        pe = rng.standard_normal((1 + grid * grid, E)).astype(np.float32)
        interp.append((name, pe, grid, gh, gw, 0.1, full))
    saddle = []
    for S in (3, 4, 5, 8):
        for k in range(3):
            base = rng.standard_normal(1024).astype(np.float32)
            cls = base + rng.standard_normal((S, 1024)).astype(np.float32) * np.float32(0.3 + 0.4 * k)
            cls *= rng.uniform(0.5, 2.0, size=(S, 1)).astype(np.float32)
            saddle.append((f"s{S}_{k}", cls.astype(np.float32)))
    return rope, interp, saddle


def sha(a):
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_da3host():
    if orc.ref_lib() is None:
        raise SystemExit("oracle/_ref could not be built: the DA3cpplib checkout is required")
    rope, interp, saddle = da3_host_cases()
    out = {}
    for name, pos, hd, freq, full in rope:
        c, s = orc.rope_tables(pos, hd, freq, impl="ref")
        if full:
            out[name + "_cos"], out[name + "_sin"] = c, s
        else:
            out[name + "_sha"] = np.array([sha(c), sha(s)])
    for name, pe, grid, gh, gw, off, full in interp:
        r = orc.interp_pos_embed(pe, grid, gh, gw, off, impl="ref")
        if full:
            out[name + "_out"] = r
        else:
            out[name + "_sha"] = np.array([sha(r)])
    for name, cls in saddle:
        out[name + "_idx"] = np.int32(orc.select_saddle(cls, impl="ref"))
    np.savez_compressed(os.path.join(HERE, "da3_host_ref.npz"), **out)


if __name__ == "__main__":
    which = sys.argv[1:] or ["preprocess", "q8", "hf", "linalg", "raypose", "nested", "da3host"]
    if "preprocess" in which:
        make_preprocess()
    if "q8" in which:
        make_q8()
    if "hf" in which:
        make_hf()
    if "linalg" in which:
        make_linalg()
    if "raypose" in which:
        make_raypose()
    if "nested" in which:
        make_nested()
    if "da3host" in which:
        make_da3host()
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))
