"""Wan2.2 VAE encode of the observation frame on B200.

Mirrors the reference interface used by the FastWAM prologue,
``self.vae.model.encode(video, self.vae.scale)`` with video [1, 3, 1, H, W]
(FastWAM/src/fastwam/models/wan22/fastwam.py:296-306; VideoVAE38_.encode,
wan22/wan_video_vae.py:1285-1304), for the first frame (T = 1), which is all
the action-chunk prologue encodes.  Parameters load from the reference's
state dict names (``encoder.*``, ``conv1.*``).

Every step runs in libfam (include/fam.h): stride-1 3x3 convolutions as the
tcgen05 GEMM's implicit convolution (``ops.conv3x3``: per tap the A rows of a
zero-bordered channels-last buffer shift by dy * (W + 2) + dx), the stride-2
ones as ``fam_vae_im2col`` + GEMM, 1x1 convolutions as GEMMs, RMS_norm(+SiLU), the AvgDown3D shortcut, the one-head
attention (scores GEMM, row softmax, P V GEMM) and the latent normalisation
as ``fam_vae_*`` kernels.  The sequence is captured once per frame size in a
CUDA graph.  With T = 1 every CausalConv3d sees two zero frames in front
(wan_video_vae.py:38-53), so its last temporal tap is packed; the temporal
downsample convs of Resample38 only fill their cache on a first chunk
(:177-190) and are not used.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Dict, List, Optional, Sequence

import torch

from . import ops
from ._lib import check, lib

Params = Dict[str, torch.Tensor]


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class _Conv:
    """Packed convolution: bf16 weight [Cout, taps * Cin_p] (K order dy, dx, c), bf16 bias."""

    def __init__(self, w: torch.Tensor, b: Optional[torch.Tensor], cin_p: int, device):
        if w.dim() == 5:                       # CausalConv3d: last temporal tap
            w = w[:, :, -1]
        cout, cin = w.shape[:2]
        self.taps = w.shape[2] * w.shape[3] if w.dim() == 4 else 1
        if w.dim() == 4:
            w = w.permute(0, 2, 3, 1)           # [Cout, kh, kw, Cin]
        w = w.reshape(cout, self.taps, cin)
        wp = torch.zeros(cout, self.taps, cin_p, dtype=torch.float32)
        wp[:, :, :cin] = w.float()
        self.w = wp.reshape(cout, self.taps * cin_p).to(device=device, dtype=torch.bfloat16).contiguous()
        self.b = None if b is None else b.reshape(-1).to(device=device, dtype=torch.bfloat16).contiguous()
        self.cout, self.cin_p = cout, cin_p


class VideoVAE38Encoder:
    """VideoVAE38_ encoder side (Encoder3d_38 + conv1) for one frame."""

    def __init__(self, state_dict: Params, dim: int = 160, z_dim: int = 48,
                 dim_mult: Sequence[int] = (1, 2, 4, 4), num_res_blocks: int = 2,
                 temperal_downsample: Sequence[bool] = (False, True, True), device="cuda"):
        self.device = torch.device(device)
        self.dim, self.z_dim = dim, z_dim
        self.dim_mult, self.num_res_blocks = tuple(dim_mult), num_res_blocks
        self.temperal_downsample = tuple(temperal_downsample)
        sd = state_dict
        dev = self.device

        def g(name):  # RMS_norm gamma as bf16 [C]
            return sd[name + ".gamma"].reshape(-1).to(device=dev, dtype=torch.bfloat16).contiguous()

        def conv(name, cin_p):
            return _Conv(sd[name + ".weight"], sd.get(name + ".bias"), cin_p, dev)

        dims = [dim * u for u in (1,) + self.dim_mult]
        for c in dims + [2 * z_dim]:
            if c % 8:
                raise ValueError(f"channel count {c} is not a multiple of 8")
        c64 = lambda c: (c + 63) // 64 * 64           # implicit convolutions: whole 64-channel K blocks per tap
        self._c64 = c64
        conv = lambda name, cin_p: _Conv(sd[name + ".weight"], sd.get(name + ".bias"), cin_p, dev)
        self.conv_in = conv("encoder.conv1", 64)      # patchified 12 channels (16 in the buffer)
        self.blocks = []
        n = len(self.dim_mult)
        for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
            pre = f"encoder.downsamples.{i}.downsamples"
            rbs, cin = [], din
            for j in range(num_res_blocks):
                rbs.append(self._res_block(sd, f"{pre}.{j}", cin, dout, g, conv))
                cin = dout
            down = i != n - 1
            t_down = self.temperal_downsample[i] if i < len(self.temperal_downsample) else False
            self.blocks.append(dict(rbs=rbs, din=din, dout=dout, down=down, ft=2 if t_down else 1,
                                    resample=conv(f"{pre}.{num_res_blocks}.resample.1", dout) if down else None))
        c = dims[-1]
        self.mid0 = self._res_block(sd, "encoder.middle.0", c, c, g, conv)
        self.attn = dict(gamma=g("encoder.middle.1.norm"), qkv=conv("encoder.middle.1.to_qkv", c),
                         proj=conv("encoder.middle.1.proj", c))
        self.mid2 = self._res_block(sd, "encoder.middle.2", c, c, g, conv)
        self.head_gamma = g("encoder.head.0")
        self.head = conv("encoder.head.2", c64(c))
        self.conv1 = conv("conv1", 2 * z_dim)
        self._bufs = {}
        self._graphs = {}

    def _res_block(self, sd, pre, cin, cout, g, conv):
        c64 = self._c64
        return dict(cin=cin, cout=cout, g0=g(pre + ".residual.0"), c1=conv(pre + ".residual.2", c64(cin)),
                    g1=g(pre + ".residual.3"), c2=conv(pre + ".residual.6", c64(cout)),
                    sc=conv(pre + ".shortcut", cin) if (pre + ".shortcut.weight") in sd else None)

    # ------------------------------------------------------------- buffers
    def _alloc(self, H: int, W: int):
        key = (H, W)
        if key in self._bufs:
            return self._bufs[key]
        if H % 16 or W % 16:
            raise ValueError(f"frame {H}x{W}: height and width must be multiples of 16")
        if ((H // 16) * (W // 16)) % 8:
            raise ValueError(f"frame {H}x{W}: the latent grid must hold a multiple of 8 positions "
                             "(the attention P V product runs over them as GEMM K)")
        dims = [self.dim * u for u in (1,) + self.dim_mult]
        h, w = H // 2, W // 2
        pmax = h * w
        cmax = max(dims + [2 * self.z_dim, 16])
        dev = self.device
        # zero-bordered conv inputs, one per resolution, rows as wide as the
        # widest input channel count there (the border is never written);
        # im2col only for the stride-2 resample convolutions
        tp, col, hh, ww, cins = {}, 8, h, w, [16]
        for blk in self.blocks:
            cins += [blk["din"], blk["dout"]]
            if blk["down"]:
                tp[(hh, ww)] = max(cins)
                hh, ww = hh // 2, ww // 2
                col = max(col, 9 * blk["dout"] * hh * ww)
                cins = [blk["dout"]]
        tp[(hh, ww)] = max(cins + [dims[-1]])
        tp = {k: torch.zeros(((k[0] + 2) * (k[1] + 2), c), device=dev, dtype=torch.bfloat16) for k, c in tp.items()}
        pl = hh * ww
        # split-K partials: the largest of every GEMM the encode issues
        part = 4
        for (m, n, k, mo) in self._gemm_shapes(H, W):
            if n % 4 == 0:
                part = max(part, self._splits(m, n, k) * mo * n)
        f32 = lambda n: torch.empty(n, device=dev, dtype=torch.float32)
        b16 = lambda n: torch.empty(n, device=dev, dtype=torch.bfloat16)
        c = dims[-1]
        bufs = dict(
            image=b16(3 * H * W), col=b16(col), tp=tp, part=f32(part),
            x=[f32(pmax * cmax) for _ in range(3)], y=f32(pmax * cmax), xin=f32(pmax * cmax),
            raw=b16(pmax * cmax), t=b16(pl * c),
            qkv=b16(pl * 3 * c), s=f32(pl * pl), pm=b16(pl * pl), vt=b16(c * pl), o=b16(pl * c),
            z=f32(pl * 2 * self.z_dim), mu=f32(pl * 2 * self.z_dim),
            mean=f32(self.z_dim), inv_std=f32(self.z_dim), out=f32(self.z_dim * pl),
        )
        self._bufs[key] = bufs
        return bufs

    def _gemm_shapes(self, H: int, W: int):
        """(M, N, K, output rows) of every split-capable GEMM of one encode, in order."""
        c64 = self._c64
        h, w = H // 2, W // 2
        out = [(h * (w + 2), self.dim, 9 * 64, h * w)]                   # conv_in
        def rb_shapes(cin, cout):
            r = [(h * (w + 2), cout, 9 * c64(cin), h * w), (h * (w + 2), cout, 9 * c64(cout), h * w)]
            if cin != cout:
                r.append((h * w, cout, cin, h * w))                       # 1x1 shortcut
            return r
        for blk in self.blocks:
            cin = blk["din"]
            for _ in blk["rbs"]:
                out += rb_shapes(cin, blk["dout"])
                cin = blk["dout"]
            if blk["down"]:
                h, w = h // 2, w // 2
                out.append((h * w, blk["dout"], 9 * blk["dout"], h * w))  # stride-2 resample (im2col)
        c, z2 = self.dim * self.dim_mult[-1], 2 * self.z_dim
        out += rb_shapes(c, c) + [(h * w, c, c, h * w)] + rb_shapes(c, c)  # middle, attention proj
        out += [(h * (w + 2), z2, 9 * c64(c), h * w), (h * w, z2, z2, h * w)]  # head, conv1
        return out

    # ----------------------------------------------------------- pieces
    @staticmethod
    def _m(buf: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
        return buf[: rows * cols].view(rows, cols)

    @staticmethod
    def _splits(M: int, N: int, K: int) -> int:
        """Split-K factor for a convolution GEMM with fewer 128 x 256 tiles than
        half the SMs (the low-resolution layers): fill about one wave."""
        tiles = ((M + 127) // 128) * ((N + 255) // 256)
        if tiles * 2 > 148:
            return 1
        return max(1, min(148 // tiles, (K + 63) // 64 // 4))

    def _gemm(self, bufs, a, cv: "_Conv", out=None, residual=None):
        """out = a W^T + b (fp32 store) or residual += a W^T + b."""
        M, K = a.shape
        N = cv.cout
        sp = self._splits(M, N, K) if N % 4 == 0 else 1
        if sp == 1:
            if residual is not None:
                ops.gemm(a, cv.w, bias=cv.b, residual=residual)
            else:
                ops.gemm(a, cv.w, bias=cv.b, out=out, out_dtype=torch.float32)
            return
        part = bufs["part"][: sp * M * N].view(sp, M, N)
        ops.gemm(a, cv.w, splits=sp, out=part)
        dst = residual if residual is not None else out
        check(lib().fam_vae_splitk_reduce(C.c_void_p(part.data_ptr()), sp, M, N, C.c_void_p(_ptr(cv.b)),
                                          C.c_void_p(dst.data_ptr()), dst.stride(0),
                                          1 if residual is not None else 0, _stream()), "fam_vae_splitk_reduce")

    def _rms(self, x, P, Cc, gamma, silu, out=None, raw=None, pad_w=0):
        out_ld = out.stride(0) if out is not None else Cc
        check(lib().fam_vae_rms(C.c_void_p(x.data_ptr()), Cc, P, Cc, C.c_void_p(_ptr(gamma)), 1 if silu else 0,
                                C.c_void_p(_ptr(out)), out_ld, pad_w, C.c_void_p(_ptr(raw)), Cc, _stream()),
              "fam_vae_rms")

    def _conv1(self, bufs, H, W, cin, cv: _Conv, out=None, residual=None):
        """Stride-1 3x3 convolution of the zero-bordered buffer of this resolution."""
        tp = bufs["tp"][(H, W)]
        M, N, K = H * (W + 2), cv.cout, cv.w.shape[1]
        sp = self._splits(M, N, K) if N % 4 == 0 else 1
        if sp == 1:
            dst = residual if residual is not None else out
            ops.conv3x3(tp, cin, W + 2, H, cv.w, out=dst, bias=cv.b, accumulate=residual is not None)
            return
        Mo = H * W
        part = bufs["part"][: sp * Mo * N].view(sp, Mo, N)
        ops.conv3x3(tp, cin, W + 2, H, cv.w, out=part, splits=sp)
        dst = residual if residual is not None else out
        check(lib().fam_vae_splitk_reduce(C.c_void_p(part.data_ptr()), sp, Mo, N, C.c_void_p(_ptr(cv.b)),
                                          C.c_void_p(dst.data_ptr()), dst.stride(0),
                                          1 if residual is not None else 0, _stream()), "fam_vae_splitk_reduce")

    def _conv3(self, bufs, src, H, W, cv: _Conv, stride, Ho, Wo, out=None, residual=None):
        cin = cv.cin_p
        check(lib().fam_vae_im2col(C.c_void_p(src.data_ptr()), cin, H, W, cin, stride, 1 if stride == 1 else 0,
                                   Ho, Wo, C.c_void_p(bufs["col"].data_ptr()), 9 * cin, _stream()),
              "fam_vae_im2col")
        col = self._m(bufs["col"], Ho * Wo, 9 * cin)
        self._gemm(bufs, col, cv, out=out, residual=residual)

    def _res(self, bufs, rb, xi, H, W):
        """ResidualBlock (wan_video_vae.py:267-302); returns the output stream index."""
        P, cin, cout = H * W, rb["cin"], rb["cout"]
        X = self._m(bufs["x"][xi], P, cin)
        tp = bufs["tp"][(H, W)]
        raw = self._m(bufs["raw"], P, cin) if rb["sc"] is not None else None
        self._rms(X, P, cin, rb["g0"], True, out=tp, raw=raw, pad_w=W)
        Y = self._m(bufs["y"], P, cout)
        self._conv1(bufs, H, W, cin, rb["c1"], out=Y)
        self._rms(Y, P, cout, rb["g1"], True, out=tp, pad_w=W)
        if rb["sc"] is None:
            self._conv1(bufs, H, W, cout, rb["c2"], residual=X)
            return xi
        xo = (xi + 1) % 3
        XO = self._m(bufs["x"][xo], P, cout)
        self._gemm(bufs, raw, rb["sc"], out=XO)
        self._conv1(bufs, H, W, cout, rb["c2"], residual=XO)
        return xo

    def _attention(self, bufs, xi, H, W):
        """AttentionBlock (wan_video_vae.py:304-342), one head over the frame's tokens."""
        a, P, c = self.attn, H * W, self.dim * self.dim_mult[-1]
        X = self._m(bufs["x"][xi], P, c)
        T = self._m(bufs["t"], P, c)
        self._rms(X, P, c, a["gamma"], False, out=T)
        QKV = self._m(bufs["qkv"], P, 3 * c)
        ops.gemm(T, a["qkv"].w, bias=a["qkv"].b, out=QKV)
        S = self._m(bufs["s"], P, P)
        ops.gemm(QKV[:, :c], QKV[:, c:2 * c], out=S, out_dtype=torch.float32)
        PM = self._m(bufs["pm"], P, P)
        check(lib().fam_vae_softmax(C.c_void_p(S.data_ptr()), P, P, P, 1.0 / math.sqrt(c),
                                    C.c_void_p(PM.data_ptr()), P, _stream()), "fam_vae_softmax")
        VT = self._m(bufs["vt"], c, P)
        check(lib().fam_vae_transpose(C.c_void_p(QKV[:, 2 * c:].data_ptr()), 3 * c, P, c,
                                      C.c_void_p(VT.data_ptr()), P, _stream()), "fam_vae_transpose")
        O = self._m(bufs["o"], P, c)
        ops.gemm(PM, VT, out=O)
        self._gemm(bufs, O, a["proj"], residual=X)

    def _run(self, bufs, H, W):
        h, w = H // 2, W // 2
        tp0 = bufs["tp"][(h, w)]
        check(lib().fam_vae_patchify(C.c_void_p(bufs["image"].data_ptr()), H, W, C.c_void_p(tp0.data_ptr()),
                                     tp0.stride(0), 1, _stream()), "fam_vae_patchify")
        xi = 0
        X = self._m(bufs["x"][xi], h * w, self.dim)
        self._conv1(bufs, h, w, 16, self.conv_in, out=X)
        for blk in self.blocks:
            P = h * w
            XIN = self._m(bufs["xin"], P, blk["din"])
            XIN.copy_(self._m(bufs["x"][xi], P, blk["din"]))
            for rb in blk["rbs"]:
                xi = self._res(bufs, rb, xi, h, w)
            dout = blk["dout"]
            if blk["down"]:
                X = self._m(bufs["x"][xi], P, dout)
                RAW = self._m(bufs["raw"], P, dout)
                self._rms(X, P, dout, None, False, raw=RAW)
                xd = (xi + 1) % 3
                ho, wo = h // 2, w // 2
                XD = self._m(bufs["x"][xd], ho * wo, dout)
                # ZeroPad2d((0, 1, 0, 1)) + Conv2d(3, stride 2) (wan_video_vae.py:254-258)
                self._conv3(bufs, RAW, h, w, blk["resample"], 2, ho, wo, out=XD)
                check(lib().fam_vae_avg_down_add(C.c_void_p(XIN.data_ptr()), blk["din"], h, w, blk["din"], dout,
                                                 blk["ft"], 2, C.c_void_p(XD.data_ptr()), dout, _stream()),
                      "fam_vae_avg_down_add")
                xi, h, w = xd, ho, wo
            else:
                X = self._m(bufs["x"][xi], P, dout)
                check(lib().fam_vae_avg_down_add(C.c_void_p(XIN.data_ptr()), blk["din"], h, w, blk["din"], dout,
                                                 blk["ft"], 1, C.c_void_p(X.data_ptr()), dout, _stream()),
                      "fam_vae_avg_down_add")
        xi = self._res(bufs, self.mid0, xi, h, w)
        self._attention(bufs, xi, h, w)
        xi = self._res(bufs, self.mid2, xi, h, w)
        P, c, z2 = h * w, self.dim * self.dim_mult[-1], 2 * self.z_dim
        X = self._m(bufs["x"][xi], P, c)
        self._rms(X, P, c, self.head_gamma, True, out=bufs["tp"][(h, w)], pad_w=w)
        Z = self._m(bufs["z"], P, z2)
        self._conv1(bufs, h, w, c, self.head, out=Z)
        RAW = self._m(bufs["raw"], P, z2)
        self._rms(Z, P, z2, None, False, raw=RAW)
        MU = self._m(bufs["mu"], P, z2)
        self._gemm(bufs, RAW, self.conv1, out=MU)
        check(lib().fam_vae_latent(C.c_void_p(MU.data_ptr()), z2, P, self.z_dim,
                                   C.c_void_p(bufs["mean"].data_ptr()), C.c_void_p(bufs["inv_std"].data_ptr()),
                                   C.c_void_p(bufs["out"].data_ptr()), _stream()), "fam_vae_latent")
        return h, w

    # -------------------------------------------------------------- API
    def encode(self, x: torch.Tensor, scale: List[torch.Tensor], use_graph: bool = True) -> torch.Tensor:
        """VideoVAE38_.encode(x, scale) for x [1, 3, 1, H, W] -> mu [1, z_dim, 1, H/16, W/16] (fp32)."""
        if x.dim() != 5 or x.shape[0] != 1 or x.shape[1] != 3:
            raise ValueError(f"x must be [1, 3, T, H, W], got {tuple(x.shape)}")
        if x.shape[2] != 1:
            raise NotImplementedError("only the first-frame encode (T = 1) of the action prologue is built")
        H, W = int(x.shape[3]), int(x.shape[4])
        bufs = self._alloc(H, W)
        bufs["image"].copy_(x.reshape(-1).to(device=self.device, dtype=torch.bfloat16))
        bufs["mean"].copy_(torch.as_tensor(scale[0]).reshape(-1).to(device=self.device, dtype=torch.float32))
        bufs["inv_std"].copy_(torch.as_tensor(scale[1]).reshape(-1).to(device=self.device, dtype=torch.float32))
        hl, wl = H // 16, W // 16
        if not use_graph:
            self._run(bufs, H, W)
        else:
            key = (H, W)
            g = self._graphs.get(key)
            if g is None:
                s = torch.cuda.Stream(device=self.device)
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    self._run(bufs, H, W)        # warm-up outside the capture (attributes, scratch)
                torch.cuda.current_stream().wait_stream(s)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._run(bufs, H, W)
                self._graphs[key] = g
            g.replay()
        return bufs["out"][: self.z_dim * hl * wl].view(1, self.z_dim, 1, hl, wl).clone()


def encoder_param_shapes(dim: int = 160, z_dim: int = 48, dim_mult: Sequence[int] = (1, 2, 4, 4),
                         num_res_blocks: int = 2) -> Dict[str, tuple]:
    """Names and shapes of the parameters VideoVAE38Encoder reads, as in the
    reference's VideoVAE38_ state dict (Encoder3d_38 + conv1)."""
    dims = [dim * u for u in (1,) + tuple(dim_mult)]
    s: Dict[str, tuple] = {}

    def conv(name, cout, cin, k, three_d=True):
        s[name + ".weight"] = (cout, cin, k, k, k) if three_d else (cout, cin, k, k)
        s[name + ".bias"] = (cout,)

    def rb(pre, cin, cout):
        s[pre + ".residual.0.gamma"] = (cin, 1, 1, 1)
        conv(pre + ".residual.2", cout, cin, 3)
        s[pre + ".residual.3.gamma"] = (cout, 1, 1, 1)
        conv(pre + ".residual.6", cout, cout, 3)
        if cin != cout:
            conv(pre + ".shortcut", cout, cin, 1)

    conv("encoder.conv1", dims[0], 12, 3)
    for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
        pre = f"encoder.downsamples.{i}.downsamples"
        cin = din
        for j in range(num_res_blocks):
            rb(f"{pre}.{j}", cin, dout)
            cin = dout
        if i != len(dim_mult) - 1:
            conv(f"{pre}.{num_res_blocks}.resample.1", dout, dout, 3, three_d=False)
    c = dims[-1]
    rb("encoder.middle.0", c, c)
    s["encoder.middle.1.norm.gamma"] = (c, 1, 1)
    conv("encoder.middle.1.to_qkv", 3 * c, c, 1, three_d=False)
    conv("encoder.middle.1.proj", c, c, 1, three_d=False)
    rb("encoder.middle.2", c, c)
    s["encoder.head.0.gamma"] = (c, 1, 1, 1)
    conv("encoder.head.2", 2 * z_dim, c, 3)
    conv("conv1", 2 * z_dim, 2 * z_dim, 1)
    return s


class WanVideoVAE38:
    """Holder with the reference's attributes: ``.model.encode(x, scale)``, ``.scale``,
    ``.z_dim``, ``.upsampling_factor`` (wan_video_vae.py:1347-1375)."""

    def __init__(self, state_dict: Params, mean: torch.Tensor, std: torch.Tensor, z_dim: int = 48,
                 dim: int = 160, device="cuda", **kw):
        self.model = VideoVAE38Encoder(state_dict, dim=dim, z_dim=z_dim, device=device, **kw)
        dev = torch.device(device)
        self.mean = torch.as_tensor(mean, dtype=torch.float32, device=dev)
        self.inv_std = torch.as_tensor(std, dtype=torch.float32, device=dev).reciprocal()
        self.scale = [self.mean, self.inv_std]
        self.z_dim = z_dim
        self.upsampling_factor = 16
        self.temporal_downsample_factor = 4
