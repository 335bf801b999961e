"""Write tests/golden/reference_kats.json: the known answers tensorcrate's own
tests and documentation state for the hot path, transcribed with the
file:line each comes from (paths inside the tensorcrate crate).

The reference is a Rust crate and cannot be built or run here, so its
golden values are the literal expectations in its tests and doc examples.
Each entry below restates one of them; nothing is computed from the oracle.
Run `python tests/golden/make_kats.py` to regenerate the JSON.
"""
from __future__ import annotations

import json
from pathlib import Path

NAN, INF = "nan", "inf"
NINF = "-inf"

# Constants of include/tccuda.h.
SUM, RMIN, RMAX = 0, 1, 2
FOLD, MEAN, VAR = 0, 1, 2
ADD, SUB, MUL = 0, 1, 2


def fill(value, n):
    """A run of `n` copies of `value`, kept short in the JSON."""
    return {"fill": value, "n": n}


def reduce(id_, source, dtype, shape, values, axes, kind, op, divisor, expect):
    return dict(id=id_, source=source, kind="reduce", dtype=dtype, shape=shape, input=values, axes=axes,
                reduction=kind, op=op, divisor=divisor, expect=expect)


def arg(id_, source, dtype, shape, values, axis, op, expect):
    return dict(id=id_, source=source, kind="arg", dtype=dtype, shape=shape, input=values, axis=axis, op=op,
                expect=expect)


X23 = [1.0, 5.0, 3.0, 4.0, 2.0, 6.0]
NAN33 = [1.0, NAN, 3.0, NAN, NAN, NAN, -2.0, 5.0, NAN]
TIED = [1.0, 7.0, 7.0, 2.0, -3.0, -3.0, 0.0, -3.0]
LOGITS = [0.5, 2.0, 2.0, NAN, -1.0, -3.0]


def nan_rows(length):
    """tests/broadcast_reduce.rs:815-828: three rows of 70 NaNs with a few
    numbers planted, cut to `length` per row."""
    values = [NAN] * (3 * 70)
    values[5] = 2.0
    values[69] = 2.0
    values[70 + 3] = -1.0
    values[140 + 1] = 4.0
    values[140 + 2] = 4.0
    return [v for row in range(3) for v in values[row * 70: row * 70 + length]]


def kats():
    k = []
    # src/tensors/reduction.rs:22-28 (module doc example)
    k.append(reduce("doc_sum_last", "src/tensors/reduction.rs:23", "f32", [2, 3], X23, [1], FOLD, SUM, 0,
                    [9.0, 12.0]))
    k.append(reduce("doc_max_axis0", "src/tensors/reduction.rs:24", "f32", [2, 3], X23, [0], FOLD, RMAX, 0,
                    [4.0, 5.0, 6.0]))
    k.append(reduce("doc_mean_all", "src/tensors/reduction.rs:25", "f32", [2, 3], X23, [0, 1], MEAN, 0, 0, [3.5]))
    k.append(reduce("doc_var_sample", "src/tensors/reduction.rs:26", "f32", [2, 3], X23, [1], VAR, 0, 2,
                    [4.0, 4.0]))
    k.append(arg("doc_argmax", "src/tensors/reduction.rs:27", "f32", [2, 3], X23, 1, RMAX, [1, 2]))
    # README.md:315-319
    k.append(reduce("readme_sum_all", "README.md:315", "f32", [2, 3], X23, [0, 1], FOLD, SUM, 0, [21.0]))
    k.append(reduce("readme_mean_axis0", "README.md:316", "f32", [2, 3], X23, [0], MEAN, 0, 0, [2.5, 3.5, 4.5]))
    # src/tensors/reduction.rs:261-262 (argmax doc example)
    k.append(arg("doc_logits_argmax", "src/tensors/reduction.rs:261", "f32", [2, 3], LOGITS, 1, RMAX, [1, 1]))
    # tests/broadcast_reduce.rs:506-518 extremes_pass_over_nans
    src = "tests/broadcast_reduce.rs:506-518"
    k.append(reduce("nan_max_rows", src, "f32", [3, 3], NAN33, [1], FOLD, RMAX, 0, [3.0, NINF, 5.0]))
    k.append(reduce("nan_min_rows", src, "f32", [3, 3], NAN33, [1], FOLD, RMIN, 0, [1.0, INF, -2.0]))
    k.append(reduce("nan_max_cols", src, "f32", [3, 3], NAN33, [0], FOLD, RMAX, 0, [1.0, 5.0, 3.0]))
    k.append(arg("nan_argmax_rows", src, "f32", [3, 3], NAN33, 1, RMAX, [2, 0, 1]))
    k.append(arg("nan_argmin_rows", src, "f32", [3, 3], NAN33, 1, RMIN, [0, 0, 0]))
    k.append(arg("nan_argmax_cols", src, "f32", [3, 3], NAN33, 0, RMAX, [0, 2, 0]))
    k.append(reduce("nan_sum_propagates", src, "f32", [3, 3], NAN33, [1], FOLD, SUM, 0, [NAN, NAN, NAN]))
    # tests/broadcast_reduce.rs:563-570 ties go to the first position
    src = "tests/broadcast_reduce.rs:563-570"
    k.append(arg("tied_argmax", src, "f32", [2, 4], TIED, 1, RMAX, [1, 2]))
    k.append(arg("tied_argmin", src, "f32", [2, 4], TIED, 1, RMIN, [0, 0]))
    # tests/broadcast_reduce.rs:495-503 compact sums accumulate in f32
    src = "tests/broadcast_reduce.rs:495-503"
    k.append(reduce("f16_ten_thousand_ones", src, "f16", [2, 10000], fill(1.0, 20000), [1], FOLD, SUM, 0,
                    [10000.0, 10000.0]))
    k.append(reduce("bf16_mean_of_ones", src, "bf16", [3, 1000], fill(1.0, 3000), [1], MEAN, 0, 0, [1.0, 1.0, 1.0]))
    # tests/broadcast_reduce.rs:852-863 (device variant): bf16 1000 ones down a leading axis
    k.append(reduce("bf16_column_sum", "tests/broadcast_reduce.rs:858-862", "bf16", [1000, 3], fill(1.0, 3000), [0],
                    FOLD, SUM, 0, [1000.0, 1000.0, 1000.0]))
    # tests/broadcast_reduce.rs:481-492: population variance of one element is 0
    k.append(reduce("single_population_var", "tests/broadcast_reduce.rs:489-492", "f32", [3, 1],
                    [-8.0, -1.0, 6.0], [1], VAR, 0, 1, [0.0, 0.0, 0.0]))
    # tests/broadcast_reduce.rs:815-848 NaN slices on the device
    src = "tests/broadcast_reduce.rs:815-848"
    for length in (70, 7):
        vals = nan_rows(length)
        row0_max = 2.0 if length > 5 else NINF
        k.append(reduce(f"nan_rows_{length}_max", src, "f32", [3, length], vals, [1], FOLD, RMAX, 0,
                        [row0_max, -1.0, 4.0]))
        k.append(reduce(f"nan_rows_{length}_min", src, "f32", [3, length], vals, [1], FOLD, RMIN, 0,
                        [row0_max if length > 5 else INF, -1.0, 4.0]))
        k.append(arg(f"nan_rows_{length}_argmax", src, "f32", [3, length], vals, 1, RMAX, [5, 3, 1]))
        k.append(arg(f"nan_rows_{length}_argmin", src, "f32", [3, length], vals, 1, RMIN, [5, 3, 1]))
    k.append(arg("all_nan_row_is_zero", "tests/broadcast_reduce.rs:846-848", "f32", [2, 70],
                 [NAN] * 70 + [1.0] * 70, 1, RMAX, [0, 0]))

    # src/tensors/layout.rs:512-593 (unit tests)
    src = "src/tensors/layout.rs"
    k.append(dict(id="coalesce_contiguous", source=src + ":514-518", kind="coalesce", shape=[2, 3, 4],
                  strides=[[12, 4, 1]], expect_shape=[24], expect_strides=[[1]]))
    k.append(dict(id="walk_contiguous", source=src + ":519", kind="walk", shape=[2, 3, 4], offset=5,
                  strides=[12, 4, 1], expect=list(range(5, 29))))
    k.append(dict(id="walk_transposed", source=src + ":525", kind="walk", shape=[3, 2], offset=0, strides=[1, 3],
                  expect=[0, 3, 1, 4, 2, 5]))
    k.append(dict(id="walk_scalar", source=src + ":527", kind="walk", shape=[], offset=7, strides=[], expect=[7]))
    k.append(dict(id="walk_empty", source=src + ":528", kind="walk", shape=[3, 0, 2], offset=0, strides=[0, 0, 0],
                  expect=[]))
    for left, right, want, line in [
        ([2, 3, 4], [4], [2, 3, 4], 560), ([4], [2, 3, 4], [2, 3, 4], 561), ([5, 5], [2, 3, 5, 5], [2, 3, 5, 5], 562),
        ([2, 1, 4], [3, 1], [2, 3, 4], 563), ([], [2, 3], [2, 3], 564), ([1, 0], [3, 1], [3, 0], 565),
        ([3, 4], [4, 3], None, 566), ([0], [2], None, 567),
    ]:
        k.append(dict(id=f"broadcast_shape_{line}", source=f"{src}:{line}", kind="broadcast_shape", left=left,
                      right=right, expect=want))
    for shape, strides, target, want, line in [
        ([3, 1], [1, 1], [2, 3, 4], [0, 1, 0], 569), ([4], [2], [3, 4], [0, 2], 571),
        ([2, 4], [4, 1], [4], None, 573), ([3], [1], [4], None, 574),
    ]:
        k.append(dict(id=f"broadcast_strides_{line}", source=f"{src}:{line}", kind="broadcast_strides",
                      shape=shape, strides=strides, target=target, expect=want))

    for shape, offset, strides, want, line in [([2, 3], 1, [3, 1], 7, 589), ([2, 0], 100, [3, 1], 0, 590),
                                               ([], 4, [], 5, 591)]:
        k.append(dict(id=f"reach_{line}", source=f"{src}:{line}", kind="reach", shape=shape, offset=offset,
                      strides=strides, expect=want))

    # tests/nd_tensor.rs:113-118 permutation strides; :450-457 index tensors
    k.append(dict(id="permute_strides", source="tests/nd_tensor.rs:114-117", kind="permute", shape=[2, 3, 4, 5],
                  axes=[2, 0, 3, 1], expect_shape=[4, 2, 5, 3], expect_strides=[5, 60, 1, 20]))
    k.append(dict(id="u32_transpose_copy", source="tests/nd_tensor.rs:450-454", kind="strided_copy", elem=4,
                  input=[1, 2, 3, 4, 5, 6], shape=[3, 2], offset=0, strides=[1, 3], expect=[1, 4, 2, 5, 3, 6]))
    k.append(dict(id="u32_concat_slice", source="tests/nd_tensor.rs:455-457", kind="assemble", elem=4,
                  input=[1, 2, 3, 4, 5, 6], length=10,
                  regions=[dict(shape=[2, 3], from_offset=0, from_strides=[3, 1], to_offset=0, to_strides=[5, 1]),
                           dict(shape=[2, 2], from_offset=1, from_strides=[3, 1], to_offset=3, to_strides=[5, 1])],
                  expect=[1, 2, 3, 2, 3, 4, 5, 6, 5, 6]))

    # README.md:970-978: each f16 addition rounds, 2048 + 1 = 2048
    k.append(dict(id="f16_2048_plus_1", source="README.md:975-977", kind="elementwise", dtype="f16", op=ADD,
                  a=[2048.0] * 4, b=[1.0] * 4, expect=[2048.0] * 4))

    # tests/optim.rs:34-41: SGD takes exactly the gradient step
    k.append(dict(id="sgd_exact_step", source="tests/optim.rs:34-41", kind="sgd", dtype="f32", p=[1.0, -2.0],
                  g=[0.5, 4.0], rate=0.1, expect_f32_expr=["1.0 - 0.05", "-2.0 - 0.4"]))
    # tests/optim.rs:95-100: Adam's first step is the rate, whatever the
    # gradient's magnitude (within close(): 2e-3 * (1 + |expected|))
    for mag in (0.01, 1.0, 100.0):
        k.append(dict(id=f"adam_first_step_{mag}", source="tests/optim.rs:95-100", kind="adam_first", dtype="f32",
                      rate=0.1, g=[mag], p=[0.0], expect=[-0.1], tol=2e-3 * 1.1))

    # tests/math_macro.rs:507-513: prefix_sum and sorted of small literals
    k.append(dict(id="prefix_sum_literal", source="tests/math_macro.rs:507-508", kind="prefix_sum", dtype="f32",
                  input=[1.0, 2.0, 3.0, 4.0], expect=[1.0, 3.0, 6.0, 10.0]))
    for order, want in ((0, [-1.0, 2.0, 3.0]), (1, [3.0, 2.0, -1.0])):
        k.append(dict(id=f"sorted_literal_{order}", source="tests/math_macro.rs:510-513", kind="sort", dtype="f32",
                      order=order, input_bits=None, input=[3.0, -1.0, 2.0], expect=want))
    # tests/dtypes.rs:110-116: a bf16 vector sorted descending through the trait
    k.append(dict(id="bf16_sorted_descending", source="tests/dtypes.rs:110-116", kind="sort", dtype="bf16", order=1,
                  input_bits=None, input=[1.0, 3.0, 2.0], expect=[3.0, 2.0, 1.0]))
    # tests/ordering.rs:122-135: the total order puts -NaN first, -0.0 before
    # +0.0 and +NaN last (f32::NAN is 0x7fc00000, -f32::NAN 0xffc00000)
    k.append(dict(id="sort_awkward_total_order", source="tests/ordering.rs:122-135", kind="sort", dtype="f32",
                  order=0, input_bits=[0x7FC00000, 0x00000000, 0x80000000, 0xFFC00000, 0x3F800000, 0xFF800000],
                  expect_bits={"0": 0xFFC00000, "1": 0xFF800000, "2": 0x80000000, "3": 0x00000000,
                               "5": 0x7FC00000}))

    # tests/conv.rs:54-69: correlation and convolution worked out by hand
    i33 = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0]
    taps = [1.0, 10.0, 100.0, 1000.0]
    k.append(dict(id="correlate_by_hand", source="tests/conv.rs:54-66", kind="correlate", dtype="f32",
                  shape=[3, 3], window_shape=[2, 2], flip=0, input=i33, window=taps,
                  expect=[5421.0, 6532.0, 8754.0, 9865.0]))
    k.append(dict(id="convolve_by_hand", source="tests/conv.rs:68-69", kind="correlate", dtype="f32",
                  shape=[3, 3], window_shape=[2, 2], flip=1, input=i33, window=taps,
                  expect=[1245.0, 2356.0, 4578.0, 5689.0]))
    for flip in (0, 1):
        k.append(dict(id=f"correlate_unit_window_{flip}", source="tests/conv.rs:71-80", kind="correlate",
                      dtype="f32", shape=[3, 3], window_shape=[1, 1], flip=flip, input=i33, window=[3.0],
                      expect=[3.0 * v for v in i33]))
    # tests/conv.rs:95-117: padding and flipping
    i22 = [1.0, 2.0, 3.0, 4.0]
    k.append(dict(id="pad_1_1", source="tests/conv.rs:98-106", kind="pad", dtype="f32", shape=[2, 2], pad=[1, 1],
                  input=i22, expect=[0, 0, 0, 0, 0, 1, 2, 0, 0, 3, 4, 0, 0, 0, 0, 0]))
    k.append(dict(id="pad_0_2", source="tests/conv.rs:108-113", kind="pad", dtype="f32", shape=[2, 2], pad=[0, 2],
                  input=i22, expect=[0, 0, 1, 2, 0, 0, 0, 0, 3, 4, 0, 0]))
    k.append(dict(id="pad_0_0", source="tests/conv.rs:114", kind="pad", dtype="f32", shape=[2, 2], pad=[0, 0],
                  input=i22, expect=i22))
    k.append(dict(id="flip_2x2", source="tests/conv.rs:116", kind="flip", dtype="f32", shape=[2, 2], input=i22,
                  expect=[4.0, 3.0, 2.0, 1.0]))

    # tests/statistics.rs:198-233: moments over every element; an empty
    # vector has NaN moments
    k.append(dict(id="moments_eight", source="tests/statistics.rs:199-209", kind="moments", dtype="f32",
                  input=[2.0, 4.0, 4.0, 4.0, 5.0, 5.0, 7.0, 9.0], expect=[5.0, 32.0]))
    k.append(dict(id="moments_matrix_2x2", source="tests/statistics.rs:211-212", kind="moments", dtype="f32",
                  input=[1.0, 2.0, 3.0, 4.0], expect=[2.5, 5.0]))
    k.append(dict(id="moments_single", source="tests/statistics.rs:227-229", kind="moments", dtype="f32",
                  input=[7.0], expect=[7.0, 0.0]))
    k.append(dict(id="moments_empty", source="tests/statistics.rs:232-234", kind="moments", dtype="f32",
                  input=[], expect=[NAN, NAN]))
    # tests/statistics.rs:238-252: axis moments fold the axis they name
    m34 = [1.0, 2.0, 3.0, 4.0, 10.0, 20.0, 30.0, 40.0, -1.0, -2.0, -3.0, -4.0]
    k.append(dict(id="axis_means_rows", source="tests/statistics.rs:245", kind="axis_moments", dtype="f32",
                  shape=[3, 4], axis=0, input=m34, expect_means=[2.5, 25.0, -2.5]))
    k.append(dict(id="axis_means_columns", source="tests/statistics.rs:246-249", kind="axis_moments", dtype="f32",
                  shape=[3, 4], axis=1, input=m34, expect_means_f64=[10.0 / 3.0, 20.0 / 3.0, 10.0, 40.0 / 3.0]))
    # tests/statistics.rs:82-118: published values of the standard normal
    # cdf and quantile (mean 0, stddev 1), and the quantile's edges
    for z, want in ((0.0, 0.5), (1.0, 0.8413447460685429), (-1.0, 0.1586552539314571), (1.96, 0.9750021048517795),
                    (-3.0, 0.001349898031630095)):
        k.append(dict(id=f"normal_cdf_{z}", source="tests/statistics.rs:84-99", kind="distribution", family=0,
                      statistic=1, params=[0.0, 1.0], x=z, expect_f64=want))
    for p, want in ((0.95, 1.6448536269514722), (0.975, 1.959963984540054), (0.99, 2.326347874040841),
                    (0.5, 0.0), (0.0, NINF), (1.0, INF), (1.5, NAN), (-0.5, NAN)):
        k.append(dict(id=f"normal_ppf_{p}", source="tests/statistics.rs:101-118", kind="distribution", family=0,
                      statistic=2, params=[0.0, 1.0], x=p, expect_f64=want))
    # tests/statistics.rs:182-194: the inverse Gaussian's edges
    for id_, stat, x, params, want in (("ig_cdf_at_zero", 1, 0.0, [1.0, 1.0], 0.0),
                                       ("ig_pdf_below_zero", 0, -1.0, [1.0, 1.0], 0.0),
                                       ("ig_ppf_at_zero", 2, 0.0, [1.0, 1.0], 0.0),
                                       ("ig_ppf_at_one", 2, 1.0, [1.0, 1.0], INF),
                                       ("ig_cdf_negative_mean", 1, 1.0, [-1.0, 1.0], NAN)):
        k.append(dict(id=id_, source="tests/statistics.rs:182-186", kind="distribution", family=1, statistic=stat,
                      params=params, x=x, expect_f64=want))
    k.append(dict(id="ig_cdf_extreme_shape", source="tests/statistics.rs:188-193", kind="distribution", family=1,
                  statistic=1, params=[1.0, 1e6], x=1.0, expect_f64=0.5, tol=1e-3))
    return k


def main() -> None:
    out = Path(__file__).with_name("reference_kats.json")
    out.write_text(json.dumps({"about": __doc__.strip().splitlines()[0], "kats": kats()}, indent=1) + "\n")
    print(out)


if __name__ == "__main__":
    main()
