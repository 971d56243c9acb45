"""tcgen05 descriptor encodings against the reference's own known answers (no GPU).

tests/golden/descriptor_kats.json holds every compile-time assert of
examples/tcgen05_ptxas/descriptor.rs, each builder chain rewritten from Rust syntax into the same
chain in Python. Both the product's C ABI (libptxstd's ptxstd_idesc_* / ptxstd_smem_desc* /
ptxstd_zero_mask_*) and the oracle's restatement evaluate them. The sm_103a-only absolute
leading-address assert is skipped (sm_100a has no such mode).
"""

import ctypes as C
import json
import os
import types

import pytest

from conftest import GOLDEN

KATS = json.load(open(os.path.join(GOLDEN, "descriptor_kats.json")))


def _enums(t5):
    return dict(
        H=t5.F16ElementType, E=t5.F8f6f4ElementType, Acc=t5.FloatAccumulator,
        I=t5.I8ElementType, Major=t5.Major, Sparsity=t5.Sparsity, WsMaxShift=t5.WsMaxShift,
        Mxf4K=t5.Mxf4K, Nvf4ScaleType=t5.Nvf4ScaleType, Swizzle=t5.Swizzle,
        ColumnSpan=t5.ColumnSpan)


def _product_env():
    import ptxstd.tcgen05 as t5
    D = t5.InstrDescriptor
    env = _enums(t5)
    env.update(
        F16=types.SimpleNamespace(new=D.f16, from_bits=lambda b: D(t5.MmaKind.F16, b)),
        Tf32=types.SimpleNamespace(new=D.tf32),
        F8f6f4=types.SimpleNamespace(new=D.f8f6f4),
        I8=types.SimpleNamespace(new=D.i8),
        Mxf8f6f4=types.SimpleNamespace(new=D.mxf8f6f4),
        Mxf4=types.SimpleNamespace(new=D.mxf4),
        Mxf4nvf4=types.SimpleNamespace(new=D.mxf4nvf4),
        SmemDescriptor=t5.SmemDescriptor, ZeroColumnMask=t5.ZeroColumnMask)
    return env


# Setter table of the reference (descriptor.rs:400-411): field -> (shift, width, kinds).
_ALL = {"F16", "Tf32", "F8f6f4", "I8", "Mxf8f6f4", "Mxf4", "Mxf4nvf4"}
_SETTERS = {
    "with_sparsity": (2, 1, _ALL),
    "with_sparsity_selector": (0, 2, {"F16", "Tf32"}),
    "with_saturate": (3, 1, {"I8"}),
    "with_negate_a": (13, 1, _ALL - {"I8"}),
    "with_negate_b": (14, 1, _ALL - {"I8"}),
    "with_major_a": (15, 1, {"F16", "Tf32", "F8f6f4", "I8", "Mxf8f6f4"}),
    "with_major_b": (16, 1, {"F16", "Tf32", "F8f6f4", "I8", "Mxf8f6f4"}),
    "with_max_b_shift": (30, 2, {"F16", "Tf32", "F8f6f4", "I8"}),
    "with_scale_a_id": (29, 2, {"Mxf8f6f4", "Mxf4", "Mxf4nvf4"}),
    "with_scale_b_id": (4, 2, {"Mxf8f6f4", "Mxf4", "Mxf4nvf4"}),
    "with_k": (31, 1, {"Mxf4", "Mxf4nvf4"}),
}


def _oracle_env(O):
    import ptxstd.tcgen05 as t5
    L = O.lib()

    def call(fn, *args):
        out = C.c_uint32(0) if "idesc" in fn.__name__ else C.c_uint64(0)
        assert fn(*[int(a) for a in args], C.byref(out)) == 0, (fn.__name__, args)
        return out.value

    class Idesc:
        def __init__(self, kind, bits):
            self.kind, self.bits = kind, bits

        def to_bits(self):
            return self.bits

        def __getattr__(self, name):
            shift, width, kinds = _SETTERS[name]
            assert self.kind in kinds, (self.kind, name)
            return lambda v: Idesc(self.kind, call(L.ptxo_idesc_with_field, self.bits, shift,
                                                   width, int(v)))

    class Smem:
        def __init__(self, bits):
            self.bits = bits

        def to_bits(self):
            return self.bits

        @staticmethod
        def from_shared_address(s, lbo, sbo, swz):
            return Smem(call(L.ptxo_smem_desc, s, lbo, sbo, swz))

        def with_base_offset(self, b):
            return Smem(call(L.ptxo_smem_desc_with_base_offset, self.bits, b))

        def add_start_bytes(self, b):
            return Smem(call(L.ptxo_smem_desc_add_start_bytes, self.bits, b))

    class Zm:
        def __init__(self, bits):
            self.bits = bits

        def to_bits(self):
            return self.bits

        @staticmethod
        def new(z, u):
            return Zm(call(L.ptxo_zero_mask_new, z, u))

        @staticmethod
        def from_bits(b):
            return Zm(b)

        def with_sub_mask_start(self, sub, span, cnt):
            return Zm(call(L.ptxo_zero_mask_with_sub_mask_start, self.bits, sub, span, cnt))

        def with_column_shift(self, s):
            return Zm(call(L.ptxo_zero_mask_with_column_shift, self.bits, s))

    Zm.NONE = Zm(0)

    def ns(kind, fn):
        return types.SimpleNamespace(new=lambda *a: Idesc(kind, call(fn, *a)),
                                     from_bits=lambda b: Idesc(kind, b))

    env = _enums(t5)
    env.update(F16=ns("F16", L.ptxo_idesc_f16), Tf32=ns("Tf32", L.ptxo_idesc_tf32),
               F8f6f4=ns("F8f6f4", L.ptxo_idesc_f8f6f4), I8=ns("I8", L.ptxo_idesc_i8),
               Mxf8f6f4=ns("Mxf8f6f4", L.ptxo_idesc_mxf8f6f4), Mxf4=ns("Mxf4", L.ptxo_idesc_mxf4),
               Mxf4nvf4=ns("Mxf4nvf4", L.ptxo_idesc_mxf4nvf4), SmemDescriptor=Smem,
               ZeroColumnMask=Zm)
    return env


def _run_kats(env):
    n = 0
    for it in KATS["items"]:
        if it["cfg"]:
            continue  # sm_103a-only form
        if it["kind"] == "const":
            env[it["name"]] = eval(it["expr"], {}, env)
        else:
            assert eval(it["expr"], {}, env), (it["line"], it["rust"])
            n += 1
    return n


def test_kats_product_abi(ptxstd_lib):
    assert _run_kats(_product_env()) == 41


def test_kats_oracle(oracle):
    assert _run_kats(_oracle_env(oracle)) == 41


def test_product_rejects_what_reference_asserts(ptxstd_lib):
    import ptxstd.tcgen05 as t5
    E = t5.F8f6f4ElementType
    bad = [
        lambda: t5.InstrDescriptor.f8f6f4(E.E4m3, E.E4m3, 1, 100, 128),    # M not /16
        lambda: t5.InstrDescriptor.f8f6f4(E.E4m3, E.E4m3, 1, 128, 260),    # N > 256
        lambda: t5.InstrDescriptor.mxf4nvf4(0, 64, 128),                   # block-scaled M
        lambda: t5.InstrDescriptor.mxf4(128, 64).with_major_a(1),          # no such setter
        lambda: t5.InstrDescriptor.i8(0, 1, 128, 64).with_negate_a(True),  # no negate for i8
        lambda: t5.InstrDescriptor.f16(0, 0, 1, 128, 64).with_sparsity_selector(4),
        lambda: t5.SmemDescriptor.from_shared_address(0, 8, 1024, 2),      # LBO not /16
        lambda: t5.SmemDescriptor.from_shared_address(0, 16, 0x40000, 2),  # SBO >= 256 KiB
        lambda: t5.SmemDescriptor.from_shared_address(0, 16, 1024, 2).with_base_offset(8),
        lambda: t5.SmemDescriptor.from_shared_address(0, 16, 1024, 2).add_start_bytes(8),
        lambda: t5.ZeroColumnMask.new(0, 4),
        lambda: t5.ZeroColumnMask.new(3, 4).with_sub_mask_start(4, 0, 0),
        lambda: t5.ZeroColumnMask.NONE.with_column_shift(33),
    ]
    import ptxstd
    for f in bad:
        with pytest.raises(ptxstd.PtxStdError) as ei:
            f()
        assert ei.value.status == ptxstd.EINVAL
