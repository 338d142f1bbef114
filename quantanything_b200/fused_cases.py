"""The kernel-level benchmark configurations on the fused int8 kernel.

cfg0 (one integer Linear, [256, 768] x [768, 3072]) and cfg1 (one 3x3 conv
[32, 64, 56, 56] * [128, 64, 3, 3] with the SiLU table) run through
``qa_conv_fused_dev`` -- the tcgen05 implicit-GEMM kernel with the fused
bias / requantize / table epilogue that the resident executor uses for every
contraction -- on device-resident operands.  The parity tests compare the
outputs with the reference-generated digests (``tests/golden/configs.json``);
``bench.py`` times the launches for the fused-GEMM throughput against the
int8 tensor peak.

Operands follow the reference's integer definitions (qa_kernels.cpp:59-105
for the GEMM, :108-185 for the conv, :188-228 for the requantize,
:348-358 for the table): activations are fed as raw bytes with their zero
point folded into the bias (bias - x_zp * sum(w)), weights are the
symmetric int8 values (zero point 0), the table is built like
ActivationQuantize.prepare (quant_layers.py:461-472).
"""

import ctypes

import numpy as np

from . import configs
from .resident import FusedConvDesc, choose_block_n, device_api, pad_corrections
from .utils import dequantize, quantize


def silu_table(c):
    """SiLU table of cfg1 over [qmin, qmax] (ActivationQuantize.prepare)."""
    q_in = np.arange(c.qmin, c.qmax + 1, dtype=np.int64)
    xin = dequantize(q_in.astype(np.int32), c.mid_scale, c.mid_zp)
    sig = (1.0 / (1.0 + np.exp(-xin.astype(np.float64)))).astype(np.float32)
    return quantize(np.multiply(xin, sig), c.out_scale, c.out_zp, c.qmin,
                    c.qmax).astype(np.int32)


def _fast_requant(bias, mult, shift, abssum, xmax, x_zp):
    """Host proof that the kernel's 64-bit requantize is exact (as the
    resident planner does it)."""
    bound = xmax * abssum + np.abs(bias) + abs(x_zp) * abssum
    ts = 31 + shift
    return bool(np.all((ts >= 1) & (ts <= 62)) and all(
        int(b) < (1 << 31) and abs(int(m)) < (1 << 31) and abs(int(bi)) < (1 << 31)
        and int(b) * abs(int(m)) + (1 << (int(t) - 1)) < (1 << 62)
        for b, m, t, bi in zip(bound, mult, ts, bias)))


class FusedCase:
    """One configuration's device operands, descriptor and launch."""

    def __init__(self, lib, name, device, sm_count=148):
        import torch

        self.name, self.lib, self.device = name, lib, device
        raw = device_api(lib)
        self._raw = raw
        dev = device
        if name == "cfg0":
            c = configs.linear_cfg0()
            x = c.a.astype(np.int8)                      # [M, K] raw bytes
            N, H, W, C = x.shape[0], 1, 1, x.shape[1]
            w = c.w.astype(np.int64)                     # [Cout, K]
            geo = dict(KH=1, KW=1, SH=1, SW=1, PH=0, PW=0, DH=1, DW=1, OH=1, OW=1)
            x_zp, zp, lut = c.a_zp, c.out_zp, None
            self.M, self.K = N, C
        elif name == "cfg1":
            c = configs.conv_cfg1()
            x = np.ascontiguousarray(np.transpose(c.x, (0, 2, 3, 1))).astype(np.int8)  # NHWC
            N, H, W, C = x.shape
            w = np.transpose(c.w, (0, 2, 3, 1)).reshape(c.w.shape[0], -1).astype(np.int64)
            geo = dict(KH=3, KW=3, SH=1, SW=1, PH=1, PW=1, DH=1, DW=1, OH=H, OW=W)
            x_zp, zp, lut = c.x_zp, c.mid_zp, silu_table(c)
            self.M, self.K = N * H * W, 9 * C
        else:
            raise ValueError(name)
        self.case = c
        cout, k = w.shape
        self.N_out = cout
        bn = choose_block_n(cout, self.M, C, sm_count)
        rows = -(-cout // bn) * bn
        kp = -(-k // 16) * 16
        packed = np.zeros((rows, kp), np.int8)
        packed[:cout, :k] = w
        colsum = w.sum(axis=1)
        bias = c.bias.astype(np.int64) - x_zp * colsum
        mult, shift = c.mult.astype(np.int64), c.shift.astype(np.int64)
        fast = _fast_requant(bias, mult, shift, np.abs(w).sum(axis=1), 128, x_zp)

        def put(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        self.x_dev = put(x.view(np.uint8))
        self.w_dev = put(packed)
        self.b_dev, self.m_dev, self.s_dev = put(bias), put(mult), put(shift)
        self.out_dev = torch.empty(self.M * cout, dtype=torch.uint8, device=dev)
        d = FusedConvDesc()
        d.x, d.x_pix_stride, d.x_signed, d.x_zp = self.x_dev.data_ptr(), C, 1, int(x_zp)
        d.N, d.H, d.W, d.C = N, H, W, C
        for k_, v in geo.items():
            setattr(d, k_, int(v))
        d.Cout, d.groups = cout, 1
        d.w, d.w_rows, d.w_kp = self.w_dev.data_ptr(), rows, kp
        d.bias, d.mult, d.shift = self.b_dev.data_ptr(), self.m_dev.data_ptr(), self.s_dev.data_ptr()
        d.zp, d.qmin, d.qmax, d.fast = int(zp), int(c.qmin), int(c.qmax), int(fast)
        if lut is not None:
            self.lut_dev = put(lut)
            d.lut, d.lut_offset, d.lut_len = self.lut_dev.data_ptr(), int(c.qmin), len(lut)
        d.out, d.out_pix_stride = self.out_dev.data_ptr(), cout
        d.block_n = bn
        if name == "cfg1":
            corr, rcls, ccls, ncol = pad_corrections(w.reshape(cout, 3, 3, C), x_zp, H, W, **geo)
            self.corr_dev, self.rcls_dev, self.ccls_dev = put(corr), put(rcls), put(ccls)
            d.pad_corr, d.pad_row_class = self.corr_dev.data_ptr(), self.rcls_dev.data_ptr()
            d.pad_col_class = self.ccls_dev.data_ptr()
            d.pad_col_classes, d.pad_classes = ncol, corr.shape[0]
        self.desc = d
        self.ops = 2 * self.M * cout * self.K
        self.bytes = x.nbytes + packed.nbytes + self.M * cout

    def launch(self, stream):
        rc = self._raw.qa_conv_fused_dev(ctypes.byref(self.desc), stream)
        if rc != 0:
            msg = self.lib.raw.qa_last_error().decode(errors="replace")
            raise RuntimeError(f"{self.name}: qa_conv_fused_dev failed ({rc}): {msg}")

    def output_int32(self):
        """The output in the reference's layout and dtype (int32; NCHW for
        the conv)."""
        y = self.out_dev.cpu().numpy().view(np.int8).astype(np.int32)
        if self.name == "cfg0":
            return y.reshape(self.M, self.N_out)
        n, _, h, w = self.case.x.shape
        return np.ascontiguousarray(y.reshape(n, h, w, self.N_out).transpose(0, 3, 1, 2))
