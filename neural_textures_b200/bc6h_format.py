"""BC6H block-format tables (data), and the generator of include/neural_textures/bc6h_format.h.

BC6H is the 128-bit 4x4-texel HDR block format of Direct3D 11 / the Khronos Data Format
Specification.  The 2-region partition masks are the same table the reference carries as
gBC6HPartitionSets (train.cu:20-29, one bit per texel = region), and the per-mode endpoint
precisions of the 2-region modes are its gBC6HPartitionNumBits (train.cu:31-34).  The
bit layouts below list, for every mode, the header fields in block-bit order (LSB first):
`r0[9:0]` stores bits 0..9 of endpoint 0's red channel at increasing block positions;
`r0[10:11]` (ascending) stores bit 11 first, then bit 10 (the format's reversed high bits
of modes 13 and 14).  Endpoints: 0 / 1 = region 0 (A / B), 2 / 3 = region 1 (A / B).

    python -m neural_textures_b200.bc6h_format   # rewrites include/neural_textures/bc6h_format.h
"""
from __future__ import annotations

import os
import re

# (mode bits value, mode bit count, endpoint bits, (delta r, g, b), transformed, regions, layout)
MODES = [
    (0x00, 2, 10, (5, 5, 5), True, 2,
     "g2[4] b2[4] b3[4] r0[9:0] g0[9:0] b0[9:0] r1[4:0] g3[4] g2[3:0] g1[4:0] b3[0] g3[3:0] b1[4:0] "
     "b3[1] b2[3:0] r2[4:0] b3[2] r3[4:0] b3[3]"),
    (0x01, 2, 7, (6, 6, 6), True, 2,
     "g2[5] g3[4] g3[5] r0[6:0] b3[0] b3[1] b2[4] g0[6:0] b2[5] b3[2] g2[4] b0[6:0] b3[3] b3[5] b3[4] "
     "r1[5:0] g2[3:0] g1[5:0] g3[3:0] b1[5:0] b2[3:0] r2[5:0] r3[5:0]"),
    (0x02, 5, 11, (5, 4, 4), True, 2,
     "r0[9:0] g0[9:0] b0[9:0] r1[4:0] r0[10] g2[3:0] g1[3:0] g0[10] b3[0] g3[3:0] b1[3:0] b0[10] b3[1] "
     "b2[3:0] r2[4:0] b3[2] r3[4:0] b3[3]"),
    (0x06, 5, 11, (4, 5, 4), True, 2,
     "r0[9:0] g0[9:0] b0[9:0] r1[3:0] r0[10] g3[4] g2[3:0] g1[4:0] g0[10] g3[3:0] b1[3:0] b0[10] b3[1] "
     "b2[3:0] r2[3:0] b3[0] b3[2] r3[3:0] g2[4] b3[3]"),
    (0x0A, 5, 11, (4, 4, 5), True, 2,
     "r0[9:0] g0[9:0] b0[9:0] r1[3:0] r0[10] b2[4] g2[3:0] g1[3:0] g0[10] b3[0] g3[3:0] b1[4:0] b0[10] "
     "b2[3:0] r2[3:0] b3[1] b3[2] r3[3:0] b3[4] b3[3]"),
    (0x0E, 5, 9, (5, 5, 5), True, 2,
     "r0[8:0] b2[4] g0[8:0] g2[4] b0[8:0] b3[4] r1[4:0] g3[4] g2[3:0] g1[4:0] b3[0] g3[3:0] b1[4:0] "
     "b3[1] b2[3:0] r2[4:0] b3[2] r3[4:0] b3[3]"),
    (0x12, 5, 8, (6, 5, 5), True, 2,
     "r0[7:0] g3[4] b2[4] g0[7:0] b3[2] g2[4] b0[7:0] b3[3] b3[4] r1[5:0] g2[3:0] g1[4:0] b3[0] "
     "g3[3:0] b1[4:0] b3[1] b2[3:0] r2[5:0] r3[5:0]"),
    (0x16, 5, 8, (5, 6, 5), True, 2,
     "r0[7:0] b3[0] b2[4] g0[7:0] g2[5] g2[4] b0[7:0] g3[5] b3[4] r1[4:0] g3[4] g2[3:0] g1[5:0] "
     "g3[3:0] b1[4:0] b3[1] b2[3:0] r2[4:0] b3[2] r3[4:0] b3[3]"),
    (0x1A, 5, 8, (5, 5, 6), True, 2,
     "r0[7:0] b3[1] b2[4] g0[7:0] b2[5] g2[4] b0[7:0] b3[5] b3[4] r1[4:0] g3[4] g2[3:0] g1[4:0] b3[0] "
     "g3[3:0] b1[5:0] b2[3:0] r2[4:0] b3[2] r3[4:0] b3[3]"),
    (0x1E, 5, 6, (6, 6, 6), False, 2,
     "r0[5:0] g3[4] b3[0] b3[1] b2[4] g0[5:0] g2[5] b2[5] b3[2] g2[4] b0[5:0] g3[5] b3[3] b3[5] b3[4] "
     "r1[5:0] g2[3:0] g1[5:0] g3[3:0] b1[5:0] b2[3:0] r2[5:0] r3[5:0]"),
    (0x03, 5, 10, (10, 10, 10), False, 1,
     "r0[9:0] g0[9:0] b0[9:0] r1[9:0] g1[9:0] b1[9:0]"),
    (0x07, 5, 11, (9, 9, 9), True, 1,
     "r0[9:0] g0[9:0] b0[9:0] r1[8:0] r0[10] g1[8:0] g0[10] b1[8:0] b0[10]"),
    (0x0B, 5, 12, (8, 8, 8), True, 1,
     "r0[9:0] g0[9:0] b0[9:0] r1[7:0] r0[10:11] g1[7:0] g0[10:11] b1[7:0] b0[10:11]"),
    (0x0F, 5, 16, (4, 4, 4), True, 1,
     "r0[9:0] g0[9:0] b0[9:0] r1[3:0] r0[10:15] g1[3:0] g0[10:15] b1[3:0] b0[10:15]"),
]

# 2-region partition masks (bit i = region of texel i, texels in raster order); the table
# of the format, identical to the reference's gBC6HPartitionSets (train.cu:20-29).
PARTITIONS = [
    0xCCCC, 0x8888, 0xEEEE, 0xECC8, 0xC880, 0xFEEC, 0xFEC8, 0xEC80,
    0xC800, 0xFFEC, 0xFE80, 0xE800, 0xFFE8, 0xFF00, 0xFFF0, 0xF000,
    0xF710, 0x008E, 0x7100, 0x08CE, 0x008C, 0x7310, 0x3100, 0x8CCE,
    0x088C, 0x3110, 0x6666, 0x366C, 0x17E8, 0x0FF0, 0x718E, 0x399C,
]

# anchor texel of region 1 for each partition (its index has an implicit leading 0 bit)
ANCHORS = [15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15, 15,
           15, 2, 8, 2, 2, 8, 8, 15, 2, 8, 2, 2, 8, 8, 2, 2]

WEIGHTS3 = [0, 9, 18, 27, 37, 46, 55, 64]
WEIGHTS4 = [0, 4, 9, 13, 17, 21, 26, 30, 34, 38, 43, 47, 51, 55, 60, 64]

FIELD_M = 12  # mode bit
FIELD_D = 13  # partition bit
_CH = {"r": 0, "g": 1, "b": 2}


def layout_bits(mode_index: int):
    """[(field, bit)] for every header bit of a mode, in block-bit order (bit 0 first).
    field = endpoint * 3 + channel (0..11), FIELD_M or FIELD_D."""
    val, mbits, epb, deltas, transformed, regions, text = MODES[mode_index]
    out = [(FIELD_M, b) for b in range(mbits)]
    for tok in text.split():
        m = re.fullmatch(r"([rgb])([0-3])\[(\d+)(?::(\d+))?\]", tok)
        assert m, tok
        field = int(m.group(2)) * 3 + _CH[m.group(1)]
        a = int(m.group(3))
        b = int(m.group(4)) if m.group(4) is not None else a
        if a >= b:   # [hi:lo]: stored lo first
            bits = list(range(b, a + 1))
        else:        # [lo:hi] ascending notation: stored hi first (reversed)
            bits = list(range(b, a - 1, -1))
        out += [(field, x) for x in bits]
    if regions == 2:
        out += [(FIELD_D, b) for b in range(5)]
    return out


def check_tables():
    for i, (val, mbits, epb, deltas, transformed, regions, text) in enumerate(MODES):
        bits = layout_bits(i)
        assert len(bits) == (82 if regions == 2 else 65), (i, len(bits))
        for e in range(2 * regions):
            for c in range(3):
                prec = epb if e == 0 or not transformed else deltas[c]
                if not transformed and e > 0:
                    prec = epb
                got = sorted(b for f, b in bits if f == e * 3 + c)
                assert got == list(range(prec)), (i, e, c, got, prec)
    for p, a in zip(PARTITIONS, ANCHORS):
        assert (p >> a) & 1 == 1 and p & 1 == 0


def emit_header() -> str:
    check_tables()
    lines = [
        "// GENERATED by `python -m neural_textures_b200.bc6h_format` from neural_textures_b200/bc6h_format.py.",
        "// BC6H block-format tables (Direct3D 11 / Khronos Data Format Specification) as initializer",
        "// macros, so that C code can place them in static arrays and CUDA code in __constant__ memory.",
        "#ifndef NT_BC6H_FORMAT_H",
        "#define NT_BC6H_FORMAT_H",
        "#include <stdint.h>",
        "",
        f"#define NT_BC6H_NUM_MODES {len(MODES)}",
        f"#define NT_BC6H_FIELD_M {FIELD_M}",
        f"#define NT_BC6H_FIELD_D {FIELD_D}",
        "",
        "typedef struct NtBc6hMode {",
        "    uint8_t mode_value;   /* value of the mode bits */",
        "    uint8_t mode_bits;    /* 2 or 5 */",
        "    uint8_t endpoint_bits;",
        "    uint8_t delta_bits[3];",
        "    uint8_t transformed;",
        "    uint8_t regions;",
        "    uint8_t header_bits;  /* 82 (2 regions) or 65 */",
        "} NtBc6hMode;",
        "",
        "/* NtBc6hMode[NT_BC6H_NUM_MODES] */",
        "#define NT_BC6H_MODES_INIT { \\",
    ]
    for val, mbits, epb, d, tr, reg, _ in MODES:
        lines.append(f"    {{0x{val:02X}, {mbits}, {epb}, {{{d[0]}, {d[1]}, {d[2]}}}, {int(tr)}, {reg}, "
                     f"{82 if reg == 2 else 65}}}, \\")
    lines += ["}", "", "/* uint8_t[NT_BC6H_NUM_MODES][82]: header bit k of mode m = field << 4 | bit, where field is",
              " * endpoint * 3 + channel, NT_BC6H_FIELD_M or NT_BC6H_FIELD_D; 0xFF pads the 65-bit headers */",
              "#define NT_BC6H_LAYOUT_INIT { \\"]
    for i in range(len(MODES)):
        bits = layout_bits(i)
        enc = [(f << 4) | b for f, b in bits] + [0xFF] * (82 - len(bits))
        rows = ", ".join(f"0x{x:02X}" for x in enc)
        lines.append(f"    {{{rows}}}, \\")
    lines += ["}", "",
              "/* uint16_t[32]: bit i = region of texel i */",
              "#define NT_BC6H_PARTITIONS_INIT {" + ", ".join(f"0x{p:04X}" for p in PARTITIONS) + "}",
              "/* uint8_t[32]: anchor texel of region 1 */",
              "#define NT_BC6H_ANCHORS_INIT {" + ", ".join(str(a) for a in ANCHORS) + "}",
              "#define NT_BC6H_WEIGHTS3_INIT {" + ", ".join(map(str, WEIGHTS3)) + "}",
              "#define NT_BC6H_WEIGHTS4_INIT {" + ", ".join(map(str, WEIGHTS4)) + "}",
              "", "#endif", ""]
    return "\n".join(lines)


def _runs(mode_index: int):
    """Header fields of a mode as runs (field, first block bit, first field bit, length) of
    consecutive block bits holding consecutive ascending field bits."""
    runs = []
    for k, (f, b) in enumerate(layout_bits(mode_index)):
        if f == FIELD_M:
            continue
        if runs and runs[-1][0] == f and runs[-1][1] + runs[-1][3] == k and runs[-1][2] + runs[-1][3] == b:
            runs[-1][3] += 1
        else:
            runs.append([f, k, b, 1])
    return runs


def emit_unpack() -> str:
    """CUDA device code that extracts the endpoint and partition fields of every mode with
    straight-line shifts (no table walk); generated from the same layout tables."""
    check_tables()
    out = [
        "// GENERATED by `python -m neural_textures_b200.bc6h_format` from neural_textures_b200/bc6h_format.py.",
        "// Straight-line BC6H header unpacking: one case per mode, each field assembled from runs",
        "// of consecutive block bits (lo = block bits 0..63, hi = 64..127).",
        "#pragma once",
        "#include <stdint.h>",
        "",
        "namespace nt {",
        "",
        "__device__ __forceinline__ uint32_t bc6h_bits(uint64_t lo, uint64_t hi, int k, int n)",
        "{",
        "    const uint64_t v = k >= 64 ? (hi >> (k - 64)) : (k + n <= 64 ? (lo >> k) : ((lo >> k) | (hi << (64 - k))));",
        "    return (uint32_t)(v & ((1ull << n) - 1ull));",
        "}",
        "",
        "// e[endpoint][channel] raw stored values, d partition; returns false for reserved modes",
        "__device__ __forceinline__ void bc6h_unpack_header(int mi, uint64_t lo, uint64_t hi, int (&e)[4][3], int &d)",
        "{",
        "#pragma unroll",
        "    for (int i = 0; i < 4; ++i) e[i][0] = e[i][1] = e[i][2] = 0;",
        "    d = 0;",
        "    switch (mi) {",
    ]
    for i in range(len(MODES)):
        out.append(f"    case {i}:")
        for f, k, b, n in _runs(i):
            tgt = "d" if f == FIELD_D else f"e[{f // 3}][{f % 3}]"
            shift = f" << {b}" if b else ""
            out.append(f"        {tgt} |= (int)(bc6h_bits(lo, hi, {k}, {n}){shift});")
        out.append("        break;")
    out += ["    default:", "        break;", "    }", "}", "", "}  // namespace nt", ""]
    return "\n".join(out)


def main():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = os.path.join(root, "include", "neural_textures", "bc6h_format.h")
    with open(path, "w") as f:
        f.write(emit_header())
    print(path)
    path = os.path.join(root, "neural_textures_b200", "csrc", "nt_bc6h_unpack.cuh")
    with open(path, "w") as f:
        f.write(emit_unpack())
    print(path)


if __name__ == "__main__":
    main()
