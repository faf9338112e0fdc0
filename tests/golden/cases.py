"""Golden case list shared by the fixture generator and the parity tests.

Each case names an op, magnetron shapes (dim 0 fastest), a PCG seed and the
input distributions.  Inputs are drawn in order from one seeded stream, exactly
as a reference context seeded with mag_ctx_set_prng_algorithm(ctx, PCG, seed)
draws them (magnetron/magnetron.c:1009-1012); fixtures store only outputs plus
the first values of every input (to pin the generator).
"""

UNARY_OPS = ["ABS", "NEG", "LOG", "SQR", "SQRT", "SIN", "COS", "STEP", "SOFTMAX", "SOFTMAX_DV",
             "SIGMOID", "SIGMOID_DV", "HARD_SIGMOID", "SILU", "TANH", "TANH_DV", "RELU",
             "RELU_DV", "GELU"]
SCALAR_OPS = ["ADDS", "SUBS", "MULS", "DIVS"]
BINARY_OPS = ["ADD", "SUB", "MUL", "DIV"]
REDUCE_OPS = ["SUM", "MEAN", "MIN", "MAX"]
# ops whose reference result depends on the x86 rcpps table; compared by tolerance
RCP_OPS = {"TANH", "GELU"}

UNARY_SHAPES = [(7, 3, 2), (8, 5), (13, 4, 3, 2, 1, 2), (5,), (1, 1, 1, 1, 1, 1), (64, 9), (3, 2, 2, 2, 2, 2)]
BINARY_SHAPES = [  # (x shape, y shape): y tiles into x by modulo on every dim
    ((7, 3, 2), (7, 3, 2)),
    ((8, 6, 4), (4, 3, 2)),
    ((12, 6, 4, 2, 2, 3), (3, 2, 4, 1, 2, 1)),
    ((16, 8), (16, 1)),
    ((16, 8), (1, 8)),
    ((5, 7, 9), (5, 7, 9)),
    ((6, 4, 2, 2, 4, 6), (6, 4, 2, 2, 4, 6)),
]
REDUCE_SHAPES = [(4, 1, 3, 2), (7, 3, 2), (256, 9), (5, 4, 3, 2, 2, 2), (1,)]
MATMUL_SHAPES = [(2, 2, 2), (3, 2, 1), (17, 33, 9), (32, 48, 24), (1, 64, 40), (8, 784, 10)]


def unary_dist(op):
    if op in ("LOG", "SQRT"):
        return ("u", 0.0, 4.0)  # the reference test range is U[0,1); extended, still >= 0
    return ("u", -6.0, 6.0)


def cases():
    out = []
    seed = 0x5EED0100
    for op in UNARY_OPS:
        for sh in UNARY_SHAPES:
            seed += 1
            out.append(dict(kind="unary", op=op, x=sh, seed=seed, dist=[unary_dist(op)]))
    for op in SCALAR_OPS:
        for sh in UNARY_SHAPES[:4]:
            seed += 1
            out.append(dict(kind="scalar", op=op, x=sh, seed=seed, xi=1.37 if op != "DIVS" else 0.73,
                            dist=[("u", -6.0, 6.0)]))
    for op in BINARY_OPS:
        for xs, ys in BINARY_SHAPES:
            seed += 1
            ydist = ("u", 0.5, 5.0) if op == "DIV" else ("u", -5.0, 5.0)
            out.append(dict(kind="binary", op=op, x=xs, y=ys, seed=seed, dist=[("u", -3.0, 3.0), ydist]))
    for op in REDUCE_OPS:
        for sh in REDUCE_SHAPES:
            seed += 1
            out.append(dict(kind="reduce", op=op, x=sh, seed=seed, dist=[("u", -1.0, 1.0)]))
    for (m, k, n) in MATMUL_SHAPES:
        seed += 1
        out.append(dict(kind="matmul", op="MATMUL", x=(m, k), y=(k, n), seed=seed,
                        dist=[("u", -1.0, 1.0), ("u", -1.0, 1.0)]))
    return out


def case_id(c):
    sh = "x".join(str(s) for s in c["x"])
    if "y" in c:
        sh += "_" + "x".join(str(s) for s in c["y"])
    return f'{c["kind"]}/{c["op"]}/{sh}'
