"""Transcribe the reference's known-answer tests for the strict path into JSON.

The reference is a Rust workspace that cannot be built in this image, so its
known answers are transcribed here case by case, each with the file:line of the
reference test it comes from (paths relative to the reference checkout).  The
output, reference_kats.json, pins both the CPU oracle (tests/test_oracle_kats.py)
and the CUDA provider (tests/test_gpu_kats.py).

Run:  python tests/golden/make_reference_kats.py   (rewrites reference_kats.json)
"""
import json
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))

F32_MAX = 0x7F7FFFFF
F32_MIN_NORMAL = 0x00800000
F64_MAX = 0x7FEFFFFFFFFFFFFF
F64_MIN_NORMAL = 0x0010000000000000
NEG32 = 0x80000000
NEG64 = 0x8000000000000000


def b32(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def b64(x):
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def bits(width, x):
    if isinstance(x, str):
        return x
    if isinstance(x, int):
        return hex(x)
    return hex(b32(x) if width == 32 else b64(x))


S32 = "Crates/core/scalar_checked_float/tests.rs"
S64 = "Crates/core/scalar_checked_float/f64_tests.rs"

scalar = []


def sc(cite, width, op, a, b, expect, policy=0):
    """expect: a float/int bit pattern, or a fault kind name."""
    entry = {"cite": cite, "width": width, "op": op, "a": bits(width, a), "policy": policy}
    if b is not None:
        entry["b"] = bits(width, b)
    if isinstance(expect, str) and not expect.startswith("0x"):
        entry["fault"] = expect
    else:
        entry["bits"] = bits(width, expect)
    scalar.append(entry)


# ---- binary32 ----------------------------------------------------------------
for v in (0x7F800000, 0xFF800000, 0x7F800001, 0xFFC12345):
    for op in ("add", "sub", "mul"):
        sc(f"{S32}:8-24", 32, op, v, 1.0, "InvalidFloatingOperand")
for p in (0x00000000, 0x80000000, 0x00000001, 0x007FFFFF, 0x00800000, 0x3F800000, 0x7F7FFFFF, 0x80000001,
          0xBF800000, 0xFF7FFFFF):
    exp = 0 if (p & 0x80000000 or (p << 1) & 0xFFFFFFFF == 0) else p
    sc(f"{S32}:26-49", 32, "relu", p, None, exp)
for v in (0x7F800000, 0xFF800000, 0x7F800001, 0xFFC12345):
    sc(f"{S32}:50-55", 32, "relu", v, None, "InvalidFloatingOperand")
sc(f"{S32}:56-61", 32, "relu", 1, None, "ArithmeticUnderflow", policy=1)
sc(f"{S32}:62-65", 32, "relu", 1, None, 1, policy=2)
sc(f"{S32}:70", 32, "add", 1.5, 2.25, 3.75)
sc(f"{S32}:71", 32, "sub", 1.5, 2.25, -0.75)
sc(f"{S32}:72", 32, "mul", 1.5, 2.25, 3.375)
sc(f"{S32}:73", 32, "div", 7.5, 2.5, 3.0)
sc(f"{S32}:74", 32, "div", 1.0, 3.0, 0x3EAAAAAB)
sc(f"{S32}:75-78", 32, "mul", F32_MAX, 2.0, "ArithmeticOverflow")
sc(f"{S32}:79-82", 32, "add", F32_MAX, F32_MAX, "ArithmeticOverflow")
sc(f"{S32}:90-96", 32, "div", 1, F32_MIN_NORMAL, 0x34000000, policy=2)
sc(f"{S32}:97-103", 32, "div", F32_MIN_NORMAL - 1, F32_MIN_NORMAL, 0x3F7FFFFE, policy=2)
sc(f"{S32}:104-113", 32, "div", F32_MIN_NORMAL, 1, 0x4B000000, policy=2)
sc(f"{S32}:114-123", 32, "div", 1, F32_MIN_NORMAL + 1, 0x34000000 - 2, policy=2)
sc(f"{S32}:124-130", 32, "div", 3, 2.0, 2, policy=2)
sc(f"{S32}:131-137", 32, "div", 5, 2.0, 2, policy=2)
sc(f"{S32}:138-142", 32, "div", 1, 2.0, 0, policy=2)
sc(f"{S32}:143-146", 32, "div", 1, 2.0, "ArithmeticUnderflow")
for n in (0, NEG32):
    for d in (0, NEG32):
        sc(f"{S32}:152-159", 32, "div", n, d, "DivideByZero")
sc(f"{S32}:160-163", 32, "div", 0x7F800000, 0, "InvalidFloatingOperand")
sc(f"{S32}:164-167", 32, "div", 0, 0x7FC00000, "InvalidFloatingOperand")
sc(f"{S32}:168-171", 32, "div", NEG32, 2.0, NEG32)
sc(f"{S32}:172-175", 32, "div", F32_MAX, 1, "ArithmeticOverflow")
sc(f"{S32}:208-209", 32, "mul", 1, 1.0, 1)
sc(f"{S32}:210-213", 32, "mul", 1, 0.5, "ArithmeticUnderflow")
sc(f"{S32}:214-218", 32, "mul", 1, 0.5, 0, policy=2)
sc(f"{S32}:219-224", 32, "mul", 1, 1.0, "ArithmeticUnderflow", policy=1)
sc(f"{S32}:229-233", 32, "mul", F32_MIN_NORMAL, 0x3F7FFFFF, "ArithmeticUnderflow")
sc(f"{S32}:234-240", 32, "mul", F32_MIN_NORMAL, 0x3F7FFFFF, F32_MIN_NORMAL, policy=2)
sc(f"{S32}:247-253", 32, "add", NEG32, 0, 0)
sc(f"{S32}:254-260", 32, "add", NEG32, NEG32, NEG32)
sc(f"{S32}:261-267", 32, "add", 0, NEG32, 0)
sc(f"{S32}:268-274", 32, "sub", NEG32, 0, NEG32)
sc(f"{S32}:275-281", 32, "sub", 0, NEG32, 0)
sc(f"{S32}:282-285", 32, "mul", NEG32, 2.0, NEG32)
sc(f"{S32}:291-297", 32, "add", 0, 1, "ArithmeticUnderflow", policy=1)
sc(f"{S32}:298-302", 32, "add", 1, 0, "ArithmeticUnderflow", policy=1)

# ---- binary64 ----------------------------------------------------------------
for p in (0, NEG64, 1, 0x000FFFFFFFFFFFFF, 0x0010000000000000, 0x3FF0000000000000, 0x7FEFFFFFFFFFFFFF,
          0x8000000000000001, 0xBFF0000000000000, 0xFFEFFFFFFFFFFFFF):
    exp = 0 if (p & NEG64 or p & ~NEG64 == 0) else p
    sc(f"{S64}:3-27", 64, "relu", p, None, exp)
for v in (0x7FF0000000000000, 0xFFF0000000000000, 0x7FF0000000000001, 0xFFF8123456789ABC):
    sc(f"{S64}:28-37", 64, "relu", v, None, "InvalidFloatingOperand")
sc(f"{S64}:38-42", 64, "relu", 1, None, "ArithmeticUnderflow", policy=1)
sc(f"{S64}:43-46", 64, "relu", 1, None, 1, policy=2)
sc(f"{S64}:60-61", 64, "add", 1.0, 2.0 ** -53, 1.0)
sc(f"{S64}:62-66", 64, "add", 1.0, 3.0 * 2.0 ** -53, 0x3FF0000000000002)
sc(f"{S64}:68", 64, "add", 1.0, -1.0, 0)
sc(f"{S64}:69-72", 64, "add", NEG64, NEG64, NEG64)
sc(f"{S64}:73-76", 64, "sub", NEG64, 0, NEG64)
sc(f"{S64}:77-80", 64, "add", 0, NEG64, 0)
sc(f"{S64}:85-88", 64, "mul", NEG64, 3.0, NEG64)
sc(f"{S64}:89", 64, "mul", -3.0, 0.0, NEG64)
sc(f"{S64}:90", 64, "sub", 1.25, 1.25, 0)
sc(f"{S64}:98", 64, "mul", F64_MIN_NORMAL, 0.5, 0x0008000000000000)
sc(f"{S64}:99-102", 64, "mul", F64_MIN_NORMAL, 0.5, 0x0008000000000000, policy=2)
sc(f"{S64}:103-107", 64, "mul", F64_MIN_NORMAL, 0.5, "ArithmeticUnderflow", policy=1)
sc(f"{S64}:109-112", 64, "mul", 1, 0.5, "ArithmeticUnderflow")
sc(f"{S64}:113-117", 64, "mul", 1 | NEG64, 0.5, NEG64, policy=2)
sc(f"{S64}:121-125", 64, "mul", F64_MIN_NORMAL, 0x3FEFFFFFFFFFFFFF, "ArithmeticUnderflow")
sc(f"{S64}:126-132", 64, "mul", F64_MIN_NORMAL, 0x3FEFFFFFFFFFFFFF, "ArithmeticUnderflow", policy=1)
sc(f"{S64}:133-139", 64, "mul", F64_MIN_NORMAL, 0x3FEFFFFFFFFFFFFF, F64_MIN_NORMAL, policy=2)
for inv in (0x7FF0000000000000, 0xFFF0000000000000, 0x7FF8000000000000):
    sc(f"{S64}:143-159", 64, "add", 1.0, inv, "InvalidFloatingOperand")
    sc(f"{S64}:143-159", 64, "sub", 1.0, inv, "InvalidFloatingOperand")
    sc(f"{S64}:143-159", 64, "mul", 1.0, inv, "InvalidFloatingOperand")
    sc(f"{S64}:143-159", 64, "mul", inv, 0.0, "InvalidFloatingOperand")
sc(f"{S64}:162-165", 64, "add", F64_MAX, F64_MAX, "ArithmeticOverflow")
sc(f"{S64}:166-169", 64, "mul", F64_MAX, 2.0, "ArithmeticOverflow")
sc(f"{S64}:170-173", 64, "sub", F64_MAX, F64_MAX | NEG64, "ArithmeticOverflow")
sc(f"{S64}:179-185", 64, "div", 1, F64_MIN_NORMAL, 0x3CB0000000000000, policy=2)
sc(f"{S64}:186-191", 64, "div", F64_MIN_NORMAL - 1, F64_MIN_NORMAL, 0x3FEFFFFFFFFFFFFE, policy=2)
sc(f"{S64}:192-198", 64, "div", F64_MIN_NORMAL, 1, 0x4330000000000000, policy=2)
sc(f"{S64}:199-207", 64, "div", 1, F64_MIN_NORMAL + 1, 0x3CB0000000000000 - 2, policy=2)
sc(f"{S64}:208-214", 64, "div", 3, 2.0, 2, policy=2)
sc(f"{S64}:215-221", 64, "div", 5, 2.0, 2, policy=2)
sc(f"{S64}:222-226", 64, "div", 1, 2.0, 0, policy=2)
sc(f"{S64}:227-230", 64, "div", 1, 2.0, "ArithmeticUnderflow")
for n in (0, NEG64):
    for d in (0, NEG64):
        sc(f"{S64}:235-242", 64, "div", n, d, "DivideByZero")
sc(f"{S64}:243-246", 64, "div", 0x7FF0000000000000, 0, "InvalidFloatingOperand")
sc(f"{S64}:247-250", 64, "div", 0, 0x7FF8000000000000, "InvalidFloatingOperand")
sc(f"{S64}:251-254", 64, "div", NEG64, 2.0, NEG64)
sc(f"{S64}:255-258", 64, "div", F64_MAX, 1, "ArithmeticOverflow")

# Randomized host-RNE equality streams: the oracle must equal host IEEE for
# every finite pair (overflow where the host gives infinity).
random_streams = [
    {"cite": f"{S32}:306-353", "width": 32, "ops": ["add", "sub", "mul"], "rng": "xorshift32", "seed": "0x9e3779b9",
     "pairs": 100000, "policy": 2, "skip_nonfinite": True},
    {"cite": f"{S32}:180-204", "width": 32, "ops": ["div"], "rng": "xorshift32", "seed": "0x91e10da5",
     "pairs": 50000, "policy": 2, "skip_nonfinite": True, "skip_zero_divisor": True},
    {"cite": f"{S64}:274-304", "width": 64, "ops": ["div"], "rng": "xorshift64", "seed": "0x91e10da57b3c2f19",
     "pairs": 50000, "policy": 2, "skip_nonfinite": True, "skip_zero_divisor": True},
    {"cite": f"{S64}:306-344", "width": 64, "ops": ["add", "sub", "mul"], "rng": "xorshift64_finite",
     "seed": "0x6a09e667f3bcc909", "pairs": 50000, "policy": 2},
]

# ---- tensor primitives ---------------------------------------------------------
MM = "Crates/core/dialect/tensor/reference/strict_matmul/tests.rs"
HW = "Crates/backends/cuda/tensor/strict_matmul/hardware.rs"
MSE = "Crates/core/dialect/tensor/reference/strict_mse/tests.rs"
SGD = "Crates/core/dialect/tensor/reference/strict_sgd/tests.rs"

matmul = []


def mm(cite, width, left_shape, left, right_shape, right, expect, tl=False, tr=False, policy=0):
    entry = {"cite": cite, "width": width, "left_shape": left_shape, "left": [bits(width, v) for v in left],
             "right_shape": right_shape, "right": [bits(width, v) for v in right], "transpose_left": tl,
             "transpose_right": tr, "policy": policy}
    if isinstance(expect, dict):
        entry["fault"] = expect
    else:
        entry["out"] = [bits(width, v) for v in expect]
    matmul.append(entry)


def fault(element, k, step, kind):
    return {"element_index": element, "reduction_index": k, "step": step, "kind": kind}


mm(f"{MM}:32-51", 32, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"))
mm(f"{MM}:52-58", 32, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], [1.0], policy=2)
mm(f"{MM}:62-66", 32, [1, 1], [1], [1, 1], [1.0], [1])
mm(f"{MM}:67-78", 32, [1, 1], [1], [1, 1], [1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"), policy=1)
mm(f"{MM}:79-89", 32, [1, 2], [1.0, -1.0], [2, 1], [1.0, 1.0], [0.0], policy=1)
for right in ([1.0, 1.0, -1.0], [1.0, 1.0, 0.0]):
    mm(f"{MM}:93-107", 32, [1, 3], [F32_MAX] * 3, [3, 1], right, fault(0, 1, "Add", "ArithmeticOverflow"), policy=2)
mm(f"{MM}:108-119", 32, [1, 1], [F32_MAX], [1, 1], [2.0], fault(0, 0, "Multiply", "ArithmeticOverflow"))
mm(f"{MM}:122-134", 32, [2, 2], [1.0, F32_MAX, F32_MAX, 1.0], [2, 2], [1.0, 2.0, 2.0, 2.0],
   fault(0, 1, "Multiply", "ArithmeticOverflow"))
mm(f"{MM}:137-150", 64, [2, 1], [1, 1.0], [1, 2], [0.5, 1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"),
   tl=True, tr=True)
mm(f"{MM}:151-167", 64, [2, 1], [1, 1.0], [1, 2], [0.5, 1.0], [1.0], tl=True, tr=True, policy=2)
mm(f"{MM}:168-179", 64, [1, 1], [F64_MIN_NORMAL], [1, 1], [0.5], [0x0008000000000000])
mm(f"{MM}:232-241", 32, [1, 2], [-1.0, 0x3F800001], [2, 1], [1.0, 0x3F7FFFFF], [0.0])
for inv in (0x7FC00000, 0x7F800000, 0xFF800000):
    mm(f"{MM}:242-254", 32, [1, 1], [inv], [1, 1], [0.0], fault(0, 0, "Multiply", "InvalidFloatingOperand"),
       policy=2)
mm(f"{MM}:259-271", 64, [1, 3], [F64_MAX] * 3, [3, 1], [1.0, 1.0, -1.0], fault(0, 1, "Add", "ArithmeticOverflow"))
# CUDA hardware gate (the same checked law on a device)
for tl, tr in ((False, False), (True, False), (False, True), (True, True)):
    left = [1.0, 4.0, 2.0, 5.0, 3.0, 6.0] if tl else [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    right = [7.0, 9.0, 11.0, 8.0, 10.0, 12.0] if tr else [7.0, 8.0, 9.0, 10.0, 11.0, 12.0]
    mm(f"{HW}:152-177", 32, [3, 2] if tl else [2, 3], left, [2, 3] if tr else [3, 2], right,
       [58.0, 64.0, 139.0, 154.0], tl=tl, tr=tr)
mm(f"{HW}:189-197", 32, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"))
mm(f"{HW}:198-202", 32, [1, 2], [2.0, 3.0], [2, 1], [4.0, 5.0], [23.0])
mm(f"{HW}:203-210", 32, [1, 2], [F32_MAX] * 2, [2, 1], [1.0, 1.0], fault(0, 1, "Add", "ArithmeticOverflow"))
mm(f"{HW}:211-218", 32, [1, 2], [F32_MAX] * 2, [2, 1], [2.0, -2.0], fault(0, 0, "Multiply", "ArithmeticOverflow"))
mm(f"{HW}:219-226", 32, [1, 2], [1.0, 0x7FC00000], [2, 1], [1.0, 1.0],
   fault(0, 1, "Multiply", "InvalidFloatingOperand"))
mm(f"{HW}:227-246", 32, [1, 2], [-1.0, 0x3F800001], [2, 1], [1.0, 0x3F7FFFFE], [0.0])
mm(f"{HW}:259-266", 32, [1, 1], [1], [1, 1], [1.0], [1])
mm(f"{HW}:267-272", 32, [1, 1], [NEG32], [1, 1], [1.0], [0])
mm(f"{HW}:273-286", 32, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], [1.0], policy=2)
mm(f"{HW}:287-303", 32, [1, 1], [1], [1, 1], [1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"), policy=1)
for phase in (2.0, 7.0):
    mm(f"{HW}:306-324", 32, [65, 2], [phase, 3.0] * 65, [2, 1], [1.0, 2.0], [phase + 6.0] * 65)
mm(f"{HW}:325-343", 32, [1, 3], [16777216.0, 1.0, -16777216.0], [3, 1], [1.0] * 3, [0.0])
mm(f"{HW}:344-364", 32, [2, 2], [1.0, 0x7FC00000, 0x7F800000, 1.0], [2, 1], [1.0, 1.0],
   fault(0, 1, "Multiply", "InvalidFloatingOperand"))
mm(f"{HW}:365-369", 32, [2, 2], [1.0, 2.0, 3.0, 4.0], [2, 1], [1.0, 1.0], [3.0, 7.0])
mm(f"{HW}:372-389", 64, [3, 2], [1.0, 4.0, 2.0, 5.0, 3.0, 6.0], [2, 3], [7.0, 9.0, 11.0, 8.0, 10.0, 12.0],
   [58.0, 64.0, 139.0, 154.0], tl=True, tr=True)
mm(f"{HW}:400-408", 64, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"))
mm(f"{HW}:409-413", 64, [1, 2], [2.0, 3.0], [2, 1], [4.0, 5.0], [23.0])
mm(f"{HW}:414-421", 64, [1, 2], [F64_MAX] * 2, [2, 1], [1.0, 1.0], fault(0, 1, "Add", "ArithmeticOverflow"))
mm(f"{HW}:422-429", 64, [1, 2], [F64_MAX] * 2, [2, 1], [2.0, -2.0], fault(0, 0, "Multiply", "ArithmeticOverflow"))
mm(f"{HW}:430-437", 64, [1, 2], [1.0, 0x7FF0000000000000], [2, 1], [1.0, 1.0],
   fault(0, 1, "Multiply", "InvalidFloatingOperand"))
mm(f"{HW}:438-457", 64, [1, 2], [-1.0, 0x3FF0000000000001], [2, 1], [1.0, 0x3FEFFFFFFFFFFFFE], [0.0])
mm(f"{HW}:470-477", 64, [1, 1], [1], [1, 1], [1.0], [1])
mm(f"{HW}:478-483", 64, [1, 1], [NEG64], [1, 1], [1.0], [0])
mm(f"{HW}:484-497", 64, [1, 2], [1, 1.0], [2, 1], [0.5, 1.0], [1.0], policy=2)
mm(f"{HW}:498-514", 64, [1, 1], [1], [1, 1], [1.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"), policy=1)
mm(f"{HW}:519-537", 64, [1, 3], [9007199254740992.0, 1.0, -9007199254740992.0], [3, 1], [1.0] * 3, [0.0])
for phase in (2.0, 7.0):
    mm(f"{HW}:538-558", 64, [65, 2], [phase, 3.0] * 65, [2, 1], [1.0, 2.0], [phase + 6.0] * 65)

mse = []


def ms(cite, width, prediction, target, expect, policy=0):
    entry = {"cite": cite, "width": width, "prediction": [bits(width, v) for v in prediction],
             "target": [bits(width, v) for v in target], "policy": policy}
    if isinstance(expect, dict):
        entry["fault"] = expect
    else:
        entry["out"] = bits(width, expect)
    mse.append(entry)


ms(f"{MSE}:28-35", 32, [F32_MAX], [F32_MAX | NEG32], fault(0, 0, "Subtract", "ArithmeticOverflow"))
ms(f"{MSE}:36-42", 32, [F32_MAX], [0.0], fault(0, 0, "Multiply", "ArithmeticOverflow"))
ms(f"{MSE}:43-49", 32, [1.0, 0x7FC00000], [0.0, 0.0], fault(0, 1, "Subtract", "InvalidFloatingOperand"))
ms(f"{MSE}:50-56", 32, [1], [0.0], fault(0, 0, "Multiply", "ArithmeticUnderflow"))
ms(f"{MSE}:64-74", 32, [3.0, 5.0], [1.0, 1.0], 10.0)
ms(f"{MSE}:94-107", 64, [3.0, 5.0], [1.0, 1.0], 10.0)
ms(f"{MSE}:108-120", 32, [1], [0.0], 0, policy=2)
ms(f"{MM}:272-284", 32, [1.0], [1.0], 0.0)

sgd = []


def sg(cite, width, weights, gradient, rate, expect, policy=0):
    entry = {"cite": cite, "width": width, "weights": [bits(width, v) for v in weights],
             "gradient": [bits(width, v) for v in gradient], "rate": bits(32, rate), "policy": policy}
    if isinstance(expect, dict):
        entry["fault"] = expect
    else:
        entry["out"] = [bits(width, v) for v in expect]
    sgd.append(entry)


sg(f"{SGD}:20-28", 32, [1.0], [1], 0.5, fault(0, 0, "Multiply", "ArithmeticUnderflow"))
sg(f"{SGD}:29-38", 32, [1.0], [1], 0.5, [1.0], policy=2)
sg(f"{SGD}:41-51", 32, [0.0], [1], 1.0, [0x80000001])
sg(f"{SGD}:52-62", 32, [0.0], [1], 1.0, fault(0, 0, "Multiply", "ArithmeticUnderflow"), policy=1)
sg(f"{SGD}:66-76", 32, [F32_MAX, 0.0], [F32_MAX | NEG32, F32_MAX], 2.0, fault(0, 0, "Multiply", "ArithmeticOverflow"))
sg(f"{SGD}:77-87", 32, [F32_MAX, 0x7FC00000], [F32_MAX | NEG32, F32_MAX], 1.0,
   fault(0, 0, "Subtract", "ArithmeticOverflow"))
sg(f"{SGD}:91-97", 32, [0x7FC00000], [1.0], 0.0, fault(0, 0, "Subtract", "InvalidFloatingOperand"))
sg(f"{SGD}:91-97", 32, [1.0], [0x7F800000], 0.0, fault(0, 0, "Multiply", "InvalidFloatingOperand"))
sg(f"{SGD}:91-97", 32, [0x7FC00000], [0x7FC00000], 0.0, fault(0, 0, "Multiply", "InvalidFloatingOperand"))
sg(f"{SGD}:110-117", 32, [1.0], [0x3F7FFFFF], 0x3F800001, [0.0])
sg(f"{SGD}:118-129", 32, [NEG32], [0.0], 1.0, [NEG32])
sg(f"{SGD}:133-143", 64, [3.0, NEG64], [1.0, 0.0], 0x3DCCCCCD, [3.0 - struct.unpack("<f", struct.pack("<I", 0x3DCCCCCD))[0], NEG64])
sg(f"{SGD}:144-156", 64, [3.0, NEG64], [1, 1.0], 0.5, fault(0, 0, "Multiply", "ArithmeticUnderflow"))
sg(f"{SGD}:190-202", 64, [2.0], [2.0], 0.5, [1.0])

# ---- whole strict programs (graph order, first faulting node wins) -------------
SG = "Crates/fusion-pcu/tests/backend_tensor_parity/scalable_graph/scalable_graph.rs"
programs = []
for width in (32, 64):
    for policy in (0, 2, 1):
        base = {
            "width": width, "policy": policy,
            "inputs": {
                "input": {"shape": [8, 2], "data": [1.0, 0.0] * 8},
                "transpose": {"shape": [2, 8], "data": [1.0] * 8 + [0.0] * 8},
                "weights": {"shape": [2, 128], "data": [2.0] * 128 + [-1.0] * 128},
                "target": {"shape": [8, 128], "data": [1.0] * 1024},
                "normalization": {"shape": [8, 128], "data": [1.0 / 512.0] * 1024},
            },
            "nodes": [
                ["preactivation", "matmul", "input", "weights", False, False],
                ["prediction", "relu", "preactivation"],
                ["loss", "mse", "prediction", "target"],
                ["difference", "sub", "prediction", "target"],
                ["normalized", "mul", "difference", "normalization"],
                ["derivative", "relu_backward", "preactivation", "normalized"],
                ["gradient", "matmul", "transpose", "derivative", False, False],
                ["updated", "sgd", "weights", "gradient", 0.5],
            ],
            "output": "updated",
        }
        ok = dict(json.loads(json.dumps(base)), cite=f"{SG}:22-45,79-95",
                  expect={"data": [255.0 / 128.0] * 128 + [-1.0] * 128})
        programs.append(ok)
        bad = json.loads(json.dumps(base))
        bad["inputs"]["target"]["data"][7 * 128 + 127] = "nan"
        bad["cite"] = f"{SG}:107-124"
        bad["expect"] = {"fault": {"node": "loss", "element_index": 0, "reduction_index": 1023, "step": "Subtract",
                                   "kind": "InvalidFloatingOperand"}}
        programs.append(bad)
        loss = {
            "cite": f"{SG}:46-56,100-106", "width": width, "policy": policy,
            "inputs": json.loads(json.dumps({k: base["inputs"][k] for k in ("input", "weights", "target")})),
            "nodes": [["preactivation", "matmul", "input", "weights", False, False],
                      ["prediction", "relu", "preactivation"], ["loss", "mse", "prediction", "target"]],
            "output": "loss", "expect": {"data": [1.0]},
        }
        programs.append(loss)

CT = "Crates/fusion-pcu/examples/checked-training/checked-training.rs"
programs.append({
    "cite": f"{CT}:16-24,66-72", "width": 32, "policy": 0,
    "inputs": {"input": {"shape": [2, 2], "data": [1.0, 0.0, 0.0, 1.0]},
               "weights": {"shape": [2, 1], "data": [2.0, -1.0]},
               "target": {"shape": [2, 1], "data": [1.0, 0.0]}},
    "nodes": [["preactivation", "matmul", "input", "weights", False, False],
              ["prediction", "relu", "preactivation"], ["loss", "mse", "prediction", "target"]],
    "output": "loss", "expect": {"data": [0.5]},
})
programs.append({
    "cite": f"{CT}:26-39,73-77", "width": 32, "policy": 0,
    "inputs": {"input": {"shape": [2, 2], "data": [1.0, 0.0, 0.0, 1.0]},
               "weights": {"shape": [2, 1], "data": [2.0, -1.0]},
               "target": {"shape": [2, 1], "data": [1.0, 0.0]}},
    "nodes": [["preactivation", "matmul", "input", "weights", False, False],
              ["prediction", "relu", "preactivation"], ["loss", "mse", "prediction", "target"],
              ["gradient", "gradient", "loss", "weights"], ["updated", "sgd", "weights", "gradient", 0.5]],
    "output": "updated", "expect": {"data": [1.5, -1.0]},
})
TR = "Crates/backends/cpu/examples/training/training.rs"
TS = "Crates/backends/cpu/benches/checked_tensor/source/source.rs"
programs.append({
    "cite": f"{TR}:18-30 with {TS}:52-66", "width": 64, "policy": 0,
    "inputs": {"input": {"shape": [2, 2], "data": [1.0, 2.0, 3.0, 4.0]},
               "transpose": {"shape": [2, 2], "data": [1.0, 3.0, 2.0, 4.0]},
               "weights": {"shape": [2, 1], "data": [0.5, 0.25]},
               "target": {"shape": [2, 1], "data": [0.0, 1.0]}},
    "nodes": [["activation", "matmul", "input", "weights", False, False],
              ["prediction", "relu", "activation"], ["loss", "mse", "prediction", "target"],
              ["difference", "sub", "prediction", "target"],
              ["derivative", "relu_backward", "activation", "difference"],
              ["gradient", "matmul", "transpose", "derivative", False, False],
              ["updated", "sgd", "weights", "gradient", 0.5]],
    "output": "updated", "expect": {"data": [-2.25, -3.75]},
})
GR = "Crates/fusion-pcu/tests/backend_tensor_parity/gradient/gradient.rs"
for width, big in ((32, F32_MAX), (64, F64_MAX)):
    for target in (1.0, 0.5):
        programs.append({
            "cite": f"{GR}:18-27,78-88", "width": width, "policy": 0,
            "inputs": {"input": {"shape": [1], "data": [0.0]}, "weights": {"shape": [1], "data": [big]},
                       "target": {"shape": [1], "data": [target]}},
            "nodes": [["prediction", "mul", "input", "weights"], ["loss", "mse", "prediction", "target"],
                      ["gradient", "gradient", "loss", "weights"]],
            "output": "gradient", "expect": {"data": [NEG32 if width == 32 else NEG64]},
        })
    programs.append({
        "cite": f"{GR}:29-38,89-92", "width": width, "policy": 0,
        "inputs": {"input": {"shape": [1], "data": [0.0]}, "weights": {"shape": [1], "data": [big]},
                   "target": {"shape": [1], "data": [1.0]}},
        "nodes": [["prediction", "mul", "input", "weights"], ["loss", "mse", "prediction", "target"],
                  ["gradient", "gradient", "loss", "input"]],
        "output": "gradient", "expect": {"fault_kind": "ArithmeticOverflow", "element_index": 0},
    })
    programs.append({
        "cite": f"{GR}:40-50,93-96", "width": width, "policy": 0,
        "inputs": {"input": {"shape": [1], "data": [0.0]}, "weights": {"shape": [1], "data": [big]},
                   "target": {"shape": [1], "data": [1.0]}},
        "nodes": [["checked", "div", "weights", "input"], ["prediction", "mul", "input", "weights"],
                  ["loss", "mse", "prediction", "target"], ["gradient", "gradient", "loss", "weights"]],
        "output": "gradient", "expect": {"fault_kind": "DivideByZero", "element_index": 0},
    })


def runs(values):
    """Run-length form [[bits, count], ...] keeps the fixture small."""
    out = []
    for v in values:
        if out and out[-1][0] == v:
            out[-1][1] += 1
        else:
            out.append([v, 1])
    return out


def encode_inputs(program):
    width = program["width"]
    for spec in program["inputs"].values():
        spec["runs"] = runs([bits(width, float("nan")) if v == "nan" else bits(width, v) for v in spec.pop("data")])
    if "data" in program["expect"]:
        program["expect"]["runs"] = runs([bits(width, v) for v in program["expect"].pop("data")])


for p in programs:
    encode_inputs(p)

if __name__ == "__main__":
    doc = {
        "about": "Known answers transcribed from the Fusion-PCU reference tests (paths relative to its checkout). "
                 "Values are hex bit patterns of binary32 (width 32) or binary64 (width 64). Policies: "
                 "0 IeeeAfterRounding, 1 RejectSubnormalResult, 2 AllowGradualUnderflow.",
        "generator": "tests/golden/make_reference_kats.py",
        "scalar": scalar, "random_streams": random_streams, "matmul": matmul, "mse": mse, "sgd": sgd,
        "programs": programs,
    }
    with open(os.path.join(HERE, "reference_kats.json"), "w") as fh:
        json.dump(doc, fh, indent=None, separators=(",", ":"))
    print(len(scalar), "scalar,", len(matmul), "matmul,", len(mse), "mse,", len(sgd), "sgd,", len(programs),
          "programs")
