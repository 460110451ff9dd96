"""da3cpplib_b200 — B200-native (sm_100a) depth path of DA3cpplib behind its own API.

The product is the native library ``libda3b.so`` (CUDA kernels + C++ engine +
C ABI, see include/da3b.h and include/da3cpp/). This Python package is a thin
ctypes host over that C ABI mirroring the reference's model API
(``load_model`` / ``Model.infer``), used by the tests and the benchmark. There is
no Python or CPU compute path: a missing or unloadable library raises.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

__all__ = ["Model", "load_model"]


class Model:
    """A GGUF depth model resident on one CUDA device (da3b_load)."""

    def __init__(self, gguf_path: str, device: int = 0):
        self.lib = _lib.load()
        self.ctx = self.lib.da3b_load(gguf_path.encode(), int(device))
        if not self.ctx:
            raise RuntimeError(f"da3b_load failed for {gguf_path}")
        dims = (ctypes.c_int * 10)()
        _lib.check(self.lib.da3b_model_dims(self.ctx, dims), "da3b_model_dims")
        (self.embed_dim, self.depth, self.num_heads, self.patch_size, self.cat_token, self.output_dim,
         self.has_aux, self.is_da2, self.has_sky, self.has_camera) = list(dims)

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.da_capi_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def last_error(self) -> str:
        e = self.lib.da_capi_last_error(self.ctx)
        return e.decode() if e else ""

    def processed_size(self, w, h, legacy=False):
        oh, ow, nr = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.check(self.lib.da3b_processed_size(self.ctx, w, h, int(legacy), ctypes.byref(oh), ctypes.byref(ow),
                                                ctypes.byref(nr)), "da3b_processed_size")
        return oh.value, ow.value, bool(nr.value)

    def infer(self, rgb: np.ndarray, views_per_scene: int = 1, rays: bool = False):
        """rgb uint8 [n][h][w][3] (host) at the processed size -> dict of numpy outputs."""
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        if rgb.ndim == 3:
            rgb = rgb[None]
        n, h, w, _ = rgb.shape
        depth = np.empty((n, h, w), np.float32)
        conf = np.empty((n, h, w), np.float32) if self.output_dim >= 2 else None
        ray = None
        if rays:
            ray = np.empty((7, n, 8 * (h // self.patch_size), 8 * (w // self.patch_size)), np.float32)
        rc = self.lib.da3b_infer_host(self.ctx, rgb.ctypes.data, n, views_per_scene, h, w, depth.ctypes.data,
                                      conf.ctypes.data if conf is not None else None,
                                      ray.ctypes.data if ray is not None else None)
        if rc != 0:
            raise RuntimeError(f"da3b_infer_host failed ({rc}): {self.last_error}")
        out = {"depth": depth}
        if conf is not None:
            out["conf"] = conf
        if ray is not None:
            out["rays"] = ray
        if self.has_sky:
            out["sky"] = self.sky(n, h, w)
        return out

    def sky(self, n, h, w):
        """Sky plane [n][h][w] of the last run (n views at h x w; models with a sky head)."""
        out = np.empty((n, h, w), np.float32)
        rc = self.lib.da3b_last_sky(self.ctx, n, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"da3b_last_sky failed ({rc}): {self.last_error}")
        return out

    def pose(self, n):
        """Camera pose of the n views of the last run: (pose_enc [n][9], ext [n][3][4], intr [n][3][3])."""
        pe = np.empty((n, 9), np.float32)
        ext = np.empty((n, 3, 4), np.float32)
        intr = np.empty((n, 3, 3), np.float32)
        rc = self.lib.da3b_last_pose(self.ctx, n, pe.ctypes.data, ext.ctypes.data, intr.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"da3b_last_pose failed ({rc}): {self.last_error}")
        return pe, ext, intr

    def infer_prepared(self, chw: np.ndarray):
        """Normalised planar f32 images [n][3][h][w] (host) -> dict of numpy outputs
        (the input of the reference's infer_preprocessed)."""
        chw = np.ascontiguousarray(chw, dtype=np.float32)
        if chw.ndim == 3:
            chw = chw[None]
        n, _, h, w = chw.shape
        depth = np.empty((n, h, w), np.float32)
        conf = np.empty((n, h, w), np.float32) if self.output_dim >= 2 else None
        rc = self.lib.da3b_infer_prepared(self.ctx, chw.ctypes.data, n, h, w, depth.ctypes.data,
                                          conf.ctypes.data if conf is not None else None, None)
        if rc == 0:
            rc = self.lib.da3b_device_status()
        if rc != 0:
            raise RuntimeError(f"da3b_infer_prepared failed ({rc}): {self.last_error}")
        out = {"depth": depth}
        if conf is not None:
            out["conf"] = conf
        if self.has_sky:
            out["sky"] = self.sky(n, h, w)
        return out

    def infer_device(self, rgb_ptr, n, h, w, depth_ptr, conf_ptr=None, rays_ptr=None, views_per_scene=1,
                     stream=None):
        """Device-pointer variant (no synchronisation)."""
        rc = self.lib.da3b_infer_device(self.ctx, ctypes.c_void_p(rgb_ptr), n, views_per_scene, h, w,
                                        ctypes.c_void_p(depth_ptr), ctypes.c_void_p(conf_ptr) if conf_ptr else None,
                                        ctypes.c_void_p(rays_ptr) if rays_ptr else None,
                                        ctypes.c_void_p(stream) if stream else None)
        if rc != 0:
            raise RuntimeError(f"da3b_infer_device failed ({rc}): {self.last_error}")

    def ref_views(self, n):
        out = (ctypes.c_int * max(1, n))()
        k = self.lib.da3b_ref_views(self.ctx, out, n)
        return list(out)[: max(0, k)]

    def launches(self, n, h, w, views_per_scene=1, rays=False):
        return self.lib.da3b_launches(self.ctx, n, views_per_scene, h, w, int(rays))

    def feature(self, layer, rows_cap=1 << 26):
        buf = np.empty(rows_cap, np.float16)
        r, c = ctypes.c_int(), ctypes.c_int()
        rc = self.lib.da3b_debug_feature(self.ctx, layer, buf.ctypes.data, buf.size, ctypes.byref(r), ctypes.byref(c))
        if rc != 0:
            raise RuntimeError(f"da3b_debug_feature failed ({rc})")
        return buf[: r.value * c.value].reshape(r.value, c.value).astype(np.float32)

    def residual(self, layer, rows_cap=1 << 27):
        """Residual stream after ViT block `layer` of the last run, f32 [rows][embed_dim]
        (needs set_capture_residuals(True) before that run)."""
        buf = np.empty(rows_cap, np.float32)
        r, c = ctypes.c_int(), ctypes.c_int()
        rc = self.lib.da3b_debug_residual(self.ctx, layer, buf.ctypes.data, buf.size, ctypes.byref(r),
                                          ctypes.byref(c))
        if rc != 0:
            raise RuntimeError(f"da3b_debug_residual failed ({rc})")
        return buf[: r.value * c.value].reshape(r.value, c.value).copy()

    def set_capture_residuals(self, on: bool):
        _lib.check(self.lib.da3b_set_capture_residuals(self.ctx, int(on)), "da3b_set_capture_residuals")

    def set_graphs(self, on: bool):
        _lib.check(self.lib.da3b_set_graphs(self.ctx, int(on)), "da3b_set_graphs")

    def set_act_quant(self, on: bool):
        _lib.check(self.lib.da3b_set_act_quant(self.ctx, int(on)), "da3b_set_act_quant")

    def set_raw_logits(self, on: bool):
        _lib.check(self.lib.da3b_set_raw_logits(self.ctx, int(on)), "da3b_set_raw_logits")


def load_model(model_path: str, device: int = 0) -> Model:
    """Counterpart of da3::load_model (include/da3cpp/da3.h)."""
    return Model(model_path, device)
