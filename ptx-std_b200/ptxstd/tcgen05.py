"""tcgen05 descriptor builders (ptx-std src/tcgen05/descriptor.rs) over the C ABI.

The classes keep the reference's builder surface: ``InstrDescriptor.f8f6f4(a, b, d, m, n)``
(``InstrDescriptor::<{MmaKind::F8f6f4}>::new``) and chained ``with_*`` setters that return new
descriptors; ``SmemDescriptor.from_shared_address(start, lbo, sbo, swizzle)``;
``ZeroColumnMask.new(zeroed, used)``. Where the reference asserts (at compile time or run time),
these raise ``PtxStdError`` with status EINVAL.
"""

from __future__ import annotations

import ctypes as C
import enum

from . import check, lib


class MmaKind(enum.IntEnum):
    F16 = 0
    Tf32 = 1
    F8f6f4 = 2
    I8 = 3
    Mxf8f6f4 = 4
    Mxf4 = 5
    Mxf4nvf4 = 6


class Swizzle(enum.IntEnum):
    None_ = 0
    Bytes128Atom32B = 1
    Bytes128 = 2
    Bytes64 = 4
    Bytes32 = 6


class Major(enum.IntEnum):
    K = 0
    Mn = 1


class Sparsity(enum.IntEnum):
    Dense = 0
    Sparse = 1


class F16ElementType(enum.IntEnum):
    F16 = 0
    Bf16 = 1


class FloatAccumulator(enum.IntEnum):
    F16 = 0
    F32 = 1


class F8f6f4ElementType(enum.IntEnum):
    E4m3 = 0
    E5m2 = 1
    E2m3 = 3
    E3m2 = 4
    E2m1 = 5


class I8ElementType(enum.IntEnum):
    U8 = 0
    S8 = 1


class WsMaxShift(enum.IntEnum):
    None_ = 0
    Shift8 = 1
    Shift16 = 2
    Shift32 = 3


class Mxf4K(enum.IntEnum):
    K64 = 0
    K96 = 1


class Nvf4ScaleType(enum.IntEnum):
    Ue4m3 = 0
    Ue8m0 = 1
    Ue5m3 = 2


class ColumnSpan(enum.IntEnum):
    Used = 0
    Zeroed = 1


_FIELDS = {"sparsity": 0, "sparsity_selector": 1, "saturate": 2, "negate_a": 3, "negate_b": 4,
           "major_a": 5, "major_b": 6, "max_b_shift": 7, "scale_a_id": 8, "scale_b_id": 9,
           "k": 10}


class InstrDescriptor:
    """A 32-bit instruction descriptor of kind ``kind`` (descriptor.rs:383-813)."""

    def __init__(self, kind: MmaKind, bits: int):
        self.kind = MmaKind(kind)
        self.bits = bits & 0xFFFFFFFF

    def to_bits(self) -> int:
        return self.bits

    @staticmethod
    def _new(fn, what, *args) -> int:
        out = C.c_uint32(0)
        check(fn(*[int(a) for a in args], C.byref(out)), what)
        return out.value

    @classmethod
    def f16(cls, a, b, d, m, n):
        return cls(MmaKind.F16, cls._new(lib().ptxstd_idesc_f16, "idesc_f16", a, b, d, m, n))

    @classmethod
    def tf32(cls, m, n):
        return cls(MmaKind.Tf32, cls._new(lib().ptxstd_idesc_tf32, "idesc_tf32", m, n))

    @classmethod
    def f8f6f4(cls, a, b, d, m, n):
        return cls(MmaKind.F8f6f4,
                   cls._new(lib().ptxstd_idesc_f8f6f4, "idesc_f8f6f4", a, b, d, m, n))

    @classmethod
    def i8(cls, a, b, m, n):
        return cls(MmaKind.I8, cls._new(lib().ptxstd_idesc_i8, "idesc_i8", a, b, m, n))

    @classmethod
    def mxf8f6f4(cls, a, b, m, n):
        return cls(MmaKind.Mxf8f6f4,
                   cls._new(lib().ptxstd_idesc_mxf8f6f4, "idesc_mxf8f6f4", a, b, m, n))

    @classmethod
    def mxf4(cls, m, n):
        return cls(MmaKind.Mxf4, cls._new(lib().ptxstd_idesc_mxf4, "idesc_mxf4", m, n))

    @classmethod
    def mxf4nvf4(cls, scale_type, m, n):
        return cls(MmaKind.Mxf4nvf4,
                   cls._new(lib().ptxstd_idesc_mxf4nvf4, "idesc_mxf4nvf4", scale_type, m, n))

    def _with(self, field: str, value) -> "InstrDescriptor":
        out = C.c_uint32(0)
        check(lib().ptxstd_idesc_set(self.bits, int(self.kind), _FIELDS[field], int(value),
                                     C.byref(out)), f"with_{field}")
        return InstrDescriptor(self.kind, out.value)

    def with_sparsity(self, s): return self._with("sparsity", s)
    def with_sparsity_selector(self, s): return self._with("sparsity_selector", s)
    def with_saturate(self, s): return self._with("saturate", bool(s))
    def with_negate_a(self, s): return self._with("negate_a", bool(s))
    def with_negate_b(self, s): return self._with("negate_b", bool(s))
    def with_major_a(self, s): return self._with("major_a", s)
    def with_major_b(self, s): return self._with("major_b", s)
    def with_max_b_shift(self, s): return self._with("max_b_shift", s)
    def with_scale_a_id(self, s): return self._with("scale_a_id", s)
    def with_scale_b_id(self, s): return self._with("scale_b_id", s)
    def with_k(self, s): return self._with("k", s)


class SmemDescriptor:
    """A 64-bit shared memory descriptor (descriptor.rs:47-250)."""

    def __init__(self, bits: int):
        self.bits = bits & 0xFFFFFFFFFFFFFFFF

    def to_bits(self) -> int:
        return self.bits

    @classmethod
    def from_shared_address(cls, start, lbo, sbo, swizzle):
        out = C.c_uint64(0)
        check(lib().ptxstd_smem_desc(int(start), int(lbo), int(sbo), int(swizzle),
                                     C.byref(out)), "smem_desc")
        return cls(out.value)

    def with_base_offset(self, bo):
        out = C.c_uint64(0)
        check(lib().ptxstd_smem_desc_with_base_offset(self.bits, int(bo), C.byref(out)),
              "with_base_offset")
        return SmemDescriptor(out.value)

    def add_start_bytes(self, b):
        out = C.c_uint64(0)
        check(lib().ptxstd_smem_desc_add_start_bytes(self.bits, int(b), C.byref(out)),
              "add_start_bytes")
        return SmemDescriptor(out.value)


class ZeroColumnMask:
    """A 64-bit zero-column mask descriptor (descriptor.rs:820-942)."""

    def __init__(self, bits: int = 0):
        self.bits = bits & 0xFFFFFFFFFFFFFFFF

    def to_bits(self) -> int:
        return self.bits

    @classmethod
    def from_bits(cls, b):
        return cls(b)

    @classmethod
    def new(cls, zeroed, used):
        out = C.c_uint64(0)
        check(lib().ptxstd_zero_mask_new(int(zeroed), int(used), C.byref(out)), "zero_mask_new")
        return cls(out.value)

    def with_sub_mask_start(self, sub, span, count):
        out = C.c_uint64(0)
        check(lib().ptxstd_zero_mask_with_sub_mask_start(self.bits, int(sub), int(span),
                                                         int(count), C.byref(out)),
              "with_sub_mask_start")
        return ZeroColumnMask(out.value)

    def with_column_shift(self, s):
        out = C.c_uint64(0)
        check(lib().ptxstd_zero_mask_with_column_shift(self.bits, int(s), C.byref(out)),
              "with_column_shift")
        return ZeroColumnMask(out.value)


ZeroColumnMask.NONE = ZeroColumnMask(0)
