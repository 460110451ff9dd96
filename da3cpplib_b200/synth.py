"""Random-init GGUF checkpoints in DA3cpplib's weight layout, plus seeded RGB8 inputs.

The reference reads its model from a GGUF file: architecture KVs under the
``depthanything3.*`` prefix (src/da_gguf_keys.h:4-81, read at
src/model_loader.cpp:73-159) and tensors by name (src/vit_block.cpp:13-29,
src/attention.cpp:35-43, src/dpt_head.cpp:108-272). Linear weights of the ViT
blocks are Q8_0 and everything else stays f32 (src/quantize.cpp:1-47). This
module writes files with exactly those keys, names, ggml shapes and types using
gguf-py (its writer and its Q8_0 quantiser), so the reference loader, the CPU
oracle and libda3b all read the same bytes.

Initialisation (seeded NumPy default_rng): every weight, bias and LayerScale is
N(0, std) with std = 0.02; LayerNorm gammas are 1 + N(0, std) (gammas of N(0, std)
would collapse every normalised activation to ~0.02 and make outputs degenerate).
``stress=True`` (parity tests) keeps every layer's output variance alive instead:
linear and conv weights are N(0, 1/fan_in), QKV weights N(0, 2.25/fan_in) so that
attention is sharp, and LayerScale 0.1 (1 + N(0, std)), so every block changes the
residual stream by about a tenth and the attention, RoPE and every head conv move the
result measurably, while the reference's own Q8_0 activation rounding stays a few
tenths of a percent of the outputs (a LayerScale near 1 lets that rounding noise
accumulate to about 1% over the blocks); for DA2 relative models the
output stage is drawn so that relu(logit) is positive on about half of the pixels
(see the out2a/out2b comment in tensors_for). The benchmark uses the stress init of
DA2-L too, so the timed model produces a non-degenerate depth map (timing does not
depend on the values).
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CACHE = os.environ.get("DA3B_CACHE", os.path.join(ROOT, "_cache"))

GGML_F32 = 0
GGML_F16 = 1
GGML_Q8_0 = 8


@dataclasses.dataclass
class ModelSpec:
    name: str
    arch: str                    # "depthanything2" | "depthanything3"
    embed_dim: int
    depth: int
    num_heads: int
    mlp_hidden: int
    features: int
    out_channels: tuple
    out_layers: tuple
    cat_token: bool
    head_pos_embed: bool
    head_norm: bool
    output_dim: int
    pos_embed_grid: int = 37
    alt_start: int = -1
    rope_start: int = -1
    qknorm_start: int = -1
    camera_token: bool = False
    aux: bool = False
    resize_mode: str = "lower_bound"
    resize_target: int = 518
    max_depth: float = 0.0
    head_dim: int = 64
    checkpoint_name: str = ""
    sky: bool = False            # metric / mono DPT sky head (head.scratch.sky_out2*)


SPECS = {
    "da2-s": ModelSpec("da2-s", "depthanything2", 384, 12, 6, 1536, 64, (48, 96, 192, 384), (2, 5, 8, 11),
                       cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1,
                       checkpoint_name="da2-small-random"),
    "da2-b": ModelSpec("da2-b", "depthanything2", 768, 12, 12, 3072, 128, (96, 192, 384, 768), (2, 5, 8, 11),
                       cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1,
                       checkpoint_name="da2-base-random"),
    "da2-l": ModelSpec("da2-l", "depthanything2", 1024, 24, 16, 4096, 256, (256, 512, 1024, 1024), (4, 11, 17, 23),
                       cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1,
                       checkpoint_name="da2-large-random"),
    "da3-l": ModelSpec("da3-l", "depthanything3", 1024, 24, 16, 4096, 256, (256, 512, 1024, 1024), (11, 15, 19, 23),
                       cat_token=True, head_pos_embed=True, head_norm=True, output_dim=2, alt_start=8, rope_start=8,
                       qknorm_start=8, camera_token=True, aux=True, resize_mode="upper_bound", resize_target=504,
                       checkpoint_name="da3-large-random"),
    # Reduced-size test models with the same structure (fast on the CPU oracle).
    "da2-t": ModelSpec("da2-t", "depthanything2", 128, 4, 2, 256, 32, (16, 32, 64, 64), (0, 1, 2, 3),
                       cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1, pos_embed_grid=8,
                       checkpoint_name="da2-tiny-random", resize_target=112),
    "da3-t": ModelSpec("da3-t", "depthanything3", 128, 6, 2, 256, 32, (16, 32, 64, 64), (2, 3, 4, 5),
                       cat_token=True, head_pos_embed=True, head_norm=True, output_dim=2, alt_start=2, rope_start=2,
                       qknorm_start=2, camera_token=True, aux=True, pos_embed_grid=8, resize_mode="upper_bound",
                       resize_target=112, checkpoint_name="da3-tiny-random"),
    "da3-s": ModelSpec("da3-s", "depthanything3", 384, 12, 6, 1536, 64, (48, 96, 192, 384), (5, 7, 9, 11),
                       cat_token=True, head_pos_embed=True, head_norm=True, output_dim=2, alt_start=4, rope_start=4,
                       qknorm_start=4, camera_token=True, aux=True, resize_mode="upper_bound", resize_target=504,
                       checkpoint_name="da3-small-random"),
    # DA3 mono / metric DPT (plain ViT, no cat token, no head norm or UV PE, depth-only
    # main head plus the sky head); the tiny one is also the nested metric branch of the
    # tests, written with the m_vit.* / m_head.* layout.
    "da3m-t": ModelSpec("da3m-t", "depthanything3", 128, 4, 2, 256, 32, (16, 32, 64, 64), (0, 1, 2, 3),
                        cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1, sky=True,
                        pos_embed_grid=8, resize_mode="upper_bound", resize_target=112,
                        checkpoint_name="da3-mono-tiny-random"),
    "da3m-l": ModelSpec("da3m-l", "depthanything3", 1024, 24, 16, 4096, 256, (256, 512, 1024, 1024),
                        (4, 11, 17, 23), cat_token=False, head_pos_embed=False, head_norm=False, output_dim=1,
                        sky=True, resize_mode="upper_bound", resize_target=504,
                        checkpoint_name="da3-mono-large-random"),
}

IMG_MEAN = (0.485, 0.456, 0.406)
IMG_STD = (0.229, 0.224, 0.225)


def _q8_0(w: np.ndarray) -> np.ndarray:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    return quants.quantize(w.astype(np.float32), GGMLQuantizationType.Q8_0)


def tensors_for(spec: ModelSpec, seed: int, stress: bool = False):
    """Yield (name, ndarray in torch/numpy order, ggml type) for every tensor."""
    rng = np.random.default_rng(seed)
    std = 0.02
    D, F = spec.embed_dim, spec.features
    hd = spec.head_dim

    def n(*shape, s=std):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    def lw(*shape, fan_in, gain=1.0):  # weight of a linear / conv with the given fan-in
        return n(*shape, s=(gain / np.sqrt(fan_in)) if stress else std)

    def gamma(*shape):
        return (1.0 + rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    out = []
    add = lambda name, arr, t=GGML_F32: out.append((name, arr, t))
    add("vit.patch_embed.weight", lw(D, 3, 14, 14, fan_in=588))
    add("vit.patch_embed.bias", n(D))
    add("vit.cls_token", n(1, 1, D))
    add("vit.pos_embed", n(1, 1 + spec.pos_embed_grid ** 2, D))
    if spec.camera_token:
        add("vit.camera_token", n(2, D))
    add("vit.norm.weight", gamma(D))
    add("vit.norm.bias", n(D))
    for i in range(spec.depth):
        p = f"vit.blk.{i}."
        add(p + "norm1.weight", gamma(D))
        add(p + "norm1.bias", n(D))
        add(p + "attn_qkv.weight", _q8_0(lw(3 * D, D, fan_in=D, gain=1.5)), GGML_Q8_0)
        add(p + "attn_qkv.bias", n(3 * D))
        if spec.qknorm_start >= 0 and i >= spec.qknorm_start:
            add(p + "attn_qnorm.weight", gamma(hd))
            add(p + "attn_qnorm.bias", n(hd))
            add(p + "attn_knorm.weight", gamma(hd))
            add(p + "attn_knorm.bias", n(hd))
        add(p + "attn_proj.weight", _q8_0(lw(D, D, fan_in=D)), GGML_Q8_0)
        add(p + "attn_proj.bias", n(D))
        add(p + "ls1", (gamma(D) * np.float32(0.1)).astype(np.float32) if stress else n(D))
        add(p + "norm2.weight", gamma(D))
        add(p + "norm2.bias", n(D))
        add(p + "mlp_fc1.weight", _q8_0(lw(spec.mlp_hidden, D, fan_in=D)), GGML_Q8_0)
        add(p + "mlp_fc1.bias", n(spec.mlp_hidden))
        add(p + "mlp_fc2.weight", _q8_0(lw(D, spec.mlp_hidden, fan_in=spec.mlp_hidden)), GGML_Q8_0)
        add(p + "mlp_fc2.bias", n(D))
        add(p + "ls2", (gamma(D) * np.float32(0.1)).astype(np.float32) if stress else n(D))
    C = (2 if spec.cat_token else 1) * D
    oc = spec.out_channels
    if spec.head_norm:
        add("head.norm.weight", gamma(C))
        add("head.norm.bias", n(C))
    for s in range(4):
        add(f"head.proj.{s}.weight", lw(oc[s], C, 1, 1, fan_in=C))
        add(f"head.proj.{s}.bias", n(oc[s]))
    add("head.resize.0.weight", lw(oc[0], oc[0], 4, 4, fan_in=oc[0]))   # ConvTranspose2d (IC, OC, 4, 4)
    add("head.resize.0.bias", n(oc[0]))
    add("head.resize.1.weight", lw(oc[1], oc[1], 2, 2, fan_in=oc[1]))
    add("head.resize.1.bias", n(oc[1]))
    add("head.resize.3.weight", lw(oc[3], oc[3], 3, 3, fan_in=9 * oc[3]))
    add("head.resize.3.bias", n(oc[3]))
    for s in range(4):
        add(f"head.scratch.layer{s + 1}_rn.weight", lw(F, oc[s], 3, 3, fan_in=9 * oc[s]))

    def pyramid(sfx):
        for r in (4, 3, 2, 1):
            p = f"head.scratch.rn{r}{sfx}."
            units = ("rc2",) if r == 4 else ("rc1", "rc2")
            for u in units:
                for cv in ("c1", "c2"):
                    add(p + f"{u}.{cv}.weight", lw(F, F, 3, 3, fan_in=9 * F, gain=1.4))
                    add(p + f"{u}.{cv}.bias", n(F))
            add(p + "out.weight", lw(F, F, 1, 1, fan_in=F))
            add(p + "out.bias", n(F))

    pyramid("")
    add("head.scratch.out1.weight", lw(F // 2, F, 3, 3, fan_in=9 * F))
    add("head.scratch.out1.bias", n(F // 2))
    if stress and spec.arch == "depthanything2" and spec.max_depth <= 0.0:
        # DA2 relative depth is relu(logit). Random out2a/out2b weights leave the logit's
        # sign set by the large per-channel offsets of the head's features, so the depth
        # map tends to be all zero. Here out2a's 32 outputs are 16 zero-DC 3x3 filters
        # (taps summing to zero per input channel) and their negatives, and out2b weighs
        # each pair by (v, -v): the logit is then a zero-mean high-pass of the features
        # and about half the pixels have positive depth, while both relus still act
        # (dropping one would double the logit).
        w = rng.standard_normal((16, F // 2, 3, 3), dtype=np.float32) * np.float32(1.4 / np.sqrt(9 * F // 2))
        w = (w - w.mean(axis=(2, 3), keepdims=True)).astype(np.float32)
        b = n(16)
        add("head.scratch.out2a.weight", np.concatenate([w, -w]).astype(np.float32))
        add("head.scratch.out2a.bias", np.concatenate([b, -b]).astype(np.float32))
        v = n(16, s=1.0 / np.sqrt(32))
        add("head.scratch.out2b.weight", np.concatenate([v, -v]).reshape(1, 32, 1, 1).astype(np.float32))
        add("head.scratch.out2b.bias", n(1))
    else:
        add("head.scratch.out2a.weight", lw(32, F // 2, 3, 3, fan_in=9 * F // 2, gain=1.4))
        add("head.scratch.out2a.bias", n(32))
        # a depth-only head (mono / metric DPT) keeps its single logit in a range where
        # exp() gives depths of a few units rather than exp(15)
        add("head.scratch.out2b.weight", lw(spec.output_dim, 32, 1, 1, fan_in=32, gain=0.1 if spec.sky else 1.0))
        add("head.scratch.out2b.bias", n(spec.output_dim))
    if spec.aux:
        pyramid("_aux")
        chans = [F, F // 2, F, F // 2, F, F // 2]
        for i in range(5):
            add(f"head.scratch.out1_aux.{i}.weight", lw(chans[i + 1], chans[i], 3, 3, fan_in=9 * chans[i]))
            add(f"head.scratch.out1_aux.{i}.bias", n(chans[i + 1]))
        add("head.scratch.out2a_aux.weight", lw(32, F // 2, 3, 3, fan_in=9 * F // 2))
        add("head.scratch.out2a_aux.bias", n(32))
        add("head.scratch.out2_aux_ln.weight", gamma(32))
        add("head.scratch.out2_aux_ln.bias", n(32))
        add("head.scratch.out2b_aux.weight", lw(7, 32, 1, 1, fan_in=32))
        add("head.scratch.out2b_aux.bias", n(7))
    if spec.camera_token:
        # camera decoder (src/cam_pose.cpp:20-32): relu(bb0) -> relu(bb2) -> fc_t | fc_q |
        # relu(fc_fov); drawn last so every earlier tensor keeps its seeded values
        Ccam = C
        add("cam.bb0.weight", _q8_0(lw(Ccam, Ccam, fan_in=Ccam)), GGML_Q8_0)
        add("cam.bb0.bias", n(Ccam))
        add("cam.bb2.weight", _q8_0(lw(Ccam, Ccam, fan_in=Ccam)), GGML_Q8_0)
        add("cam.bb2.bias", n(Ccam))
        add("cam.fc_t.weight", _q8_0(lw(3, Ccam, fan_in=Ccam)), GGML_Q8_0)
        add("cam.fc_t.bias", n(3))
        add("cam.fc_q.weight", _q8_0(lw(4, Ccam, fan_in=Ccam)), GGML_Q8_0)
        add("cam.fc_q.bias", n(4) + np.array([0, 0, 0, 1], np.float32))
        add("cam.fc_fov.weight", _q8_0(lw(2, Ccam, fan_in=Ccam)), GGML_Q8_0)
        add("cam.fc_fov.bias", n(2) + np.float32(1.0))
    if spec.sky:
        # sky head (src/dpt_head.cpp:205-222): 3x3 feat/2 -> 32, relu, 1x1 32 -> 1
        add("head.scratch.sky_out2a.weight", lw(32, F // 2, 3, 3, fan_in=9 * F // 2, gain=1.4))
        add("head.scratch.sky_out2a.bias", n(32))
        # scaled and shifted so that relu(logit) straddles the 0.3 sky threshold
        add("head.scratch.sky_out2b.weight", lw(1, 32, 1, 1, fan_in=32, gain=0.1))
        add("head.scratch.sky_out2b.bias", n(1) - np.float32(1.2 if stress else 0.0))
    return out


def write_gguf(spec: ModelSpec, path: str, seed: int, stress: bool = False, metric_branch: bool = False) -> str:
    """metric_branch=True writes the nested metric-branch layout: structure keys under
    m_vit.* / m_head.* and tensors renamed vit.* -> m_vit.*, head.* -> m_head.*
    (src/model_loader.cpp:84-127, :146-154); the head pos-embed key is omitted."""
    import gguf
    from gguf.constants import GGMLQuantizationType

    tmp = path + ".tmp"
    w = gguf.GGUFWriter(tmp, arch="depthanything3")
    P = "depthanything3."
    V = P + ("m_vit." if metric_branch else "vit.")
    Hd = P + ("m_head." if metric_branch else "head.")
    w.add_string(P + "arch", spec.arch)
    w.add_string(P + "checkpoint_name", spec.checkpoint_name or spec.name)
    w.add_uint32(P + "patch_size", 14)
    w.add_uint32(V + "embed_dim", spec.embed_dim)
    w.add_uint32(V + "depth", spec.depth)
    w.add_uint32(V + "num_heads", spec.num_heads)
    w.add_uint32(V + "head_dim", spec.head_dim)
    w.add_uint32(V + "mlp_hidden", spec.mlp_hidden)
    w.add_string(V + "ffn_type", "mlp")
    w.add_uint32(V + "num_register_tokens", 0)
    w.add_int32(V + "alt_start", spec.alt_start)
    w.add_int32(V + "rope_start", spec.rope_start)
    w.add_int32(V + "qknorm_start", spec.qknorm_start)
    w.add_float32(V + "rope_freq", 100.0)
    w.add_bool(V + "cat_token", spec.cat_token)
    w.add_bool(V + "qkv_bias", True)
    w.add_float32(V + "ln_eps", 1e-6)
    w.add_float32(V + "interpolate_offset", 0.1)
    w.add_bool(V + "interpolate_antialias", False)
    w.add_uint32(V + "pos_embed_grid", spec.pos_embed_grid)
    w.add_array(V + "out_layers", [int(v) for v in spec.out_layers])
    w.add_array(P + "img.mean", [float(v) for v in IMG_MEAN])
    w.add_array(P + "img.std", [float(v) for v in IMG_STD])
    w.add_string(P + "img.resize_mode", spec.resize_mode)
    w.add_uint32(P + "img.resize_target", spec.resize_target)
    w.add_uint32(Hd + "features", spec.features)
    w.add_array(Hd + "out_channels", [int(v) for v in spec.out_channels])
    w.add_uint32(Hd + "output_dim", spec.output_dim)
    if not metric_branch:
        w.add_bool(Hd + "pos_embed", spec.head_pos_embed)
    w.add_float32(P + "head.max_depth", float(spec.max_depth))
    w.add_bool(P + "head.has_aux", spec.aux)
    for name, arr, t in tensors_for(spec, seed, stress):
        if metric_branch and name.startswith(("vit.", "head.")):
            name = "m_" + name
        if t == GGML_Q8_0:
            w.add_tensor(name, arr, raw_dtype=GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(tmp, path)
    return path


def model_seed(name: str) -> int:
    return 20260101 + sorted(SPECS).index(name)


def ensure_gguf(name: str, stress: bool = False, seed: int | None = None, metric_branch: bool = False) -> str:
    """Path of the cached random-init GGUF for SPECS[name] (generated on first use);
    metric_branch selects the nested metric-branch layout (m_vit.* / m_head.*)."""
    spec = SPECS[name]
    seed = model_seed(name) if seed is None else seed
    key_parts = [dataclasses.asdict(spec), seed, stress, 5] + ([1] if metric_branch else [])
    key = hashlib.sha1(json.dumps(key_parts).encode()).hexdigest()[:10]
    os.makedirs(CACHE, exist_ok=True)
    tag = ("-stress" if stress else "") + ("-mbranch" if metric_branch else "")
    path = os.path.join(CACHE, f"{name}{tag}-{key}.gguf")
    if not os.path.exists(path):
        write_gguf(spec, path, seed, stress, metric_branch)
    return path


def image(seed: int, index: int, h: int, w: int) -> np.ndarray:
    """Seeded uniform RGB8 image [h][w][3] (integers in [0, 255])."""
    rng = np.random.default_rng(seed + index)
    return rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)


IMAGE_SEED = 20260101
