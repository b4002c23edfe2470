"""Writes tests/golden/reference_kat.json: the known-answer cases of fluxrt-cpp's own tests for
this path, transcribed (inputs and expected outputs as the reference tests state them).

    python tests/golden/make_golden.py

Sources (paths inside the fluxrt-cpp project):
  gather      src/spike/test_gather_scatter.cpp:39-68   (tokens {0,2,3} of 4, dim 3)
  scatter     src/spike/test_gather_scatter.cpp:73-103  (rows {1,3}; untouched rows stay -1)
  cache       src/spike/test_spatial_cache.cu:20-93     (preprocess -> all 2; restore 1/50/9/130)
  layer_norm  src/spike/test_gather_scatter.cpp:106-133 (LayerNorm of rows 1..4 and 5..8, dim 4)
  cache_mixed src/spike/test_spatial_cache_trt.cpp:243-296 (reset + partial validity; logic
              ported at a small size: the original runs 256 text + 4096 image tokens behind a
              TensorRT engine, here 4 text + 8 image tokens with the same half split)
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    cases = {}
    # --- gather (test_gather_scatter.cpp:39-68) ---
    cases["gather"] = {
        "dim": 3,
        "src": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11],
        "indices": [0, 2, 3],
        "expected": [0, 1, 2, 6, 7, 8, 9, 10, 11],
    }
    # --- scatter (test_gather_scatter.cpp:73-103) ---
    cases["scatter"] = {
        "dim": 3,
        "seq_len": 4,
        "dst_init": -1.0,
        "src": [100, 101, 102, 200, 201, 202],
        "indices": [1, 3],
        "expected": [-1, -1, -1, 100, 101, 102, -1, -1, -1, 200, 201, 202],
    }
    # --- spatial cache (test_spatial_cache.cu:20-93) ---
    img_len, txt_len, out_ch = 4, 2, 4
    cases["cache"] = {
        "img_len": img_len,
        "txt_len": txt_len,
        "out_ch": out_ch,
        # step 1: all-zero mask with nothing valid -> preprocess flips everything to 2 (:35-47)
        "mask0": [0] * (img_len + txt_len),
        "mask0_expected": [2] * (img_len + txt_len),
        # step 2: pred 1..16 with mask all 2 -> unchanged, cache filled (:50-66)
        "pred1": [float(i + 1) for i in range(img_len * out_ch)],
        "pred1_expected": [float(i + 1) for i in range(img_len * out_ch)],
        # step 3: mask {2,2,0,1,0,2}, pred 10..160 -> (:69-87)
        "mask2": [2, 2, 0, 1, 0, 2],
        "pred2": [float((i + 1) * 10) for i in range(img_len * out_ch)],
        "pred2_checks": {"0": 1.0, "4": 50.0, "8": 9.0, "12": 130.0},
    }
    # --- mixed validity (test_spatial_cache_trt.cpp:243-296, small-size port) ---
    txt, img, half = 4, 8, 4
    n = txt + img
    cases["cache_mixed"] = {
        "txt_len": txt,
        "img_len": img,
        "out_ch": 4,
        # 3a: after reset, an all-zero mask preprocesses to all 2 (:247-258)
        "after_reset_expected": [2] * n,
        # 3b: text + first half of image = 2, rest 0, then sync_output_cache (:262-266)
        "populate_mask": [2] * (txt + half) + [0] * (img - half),
        # then an all-zero mask preprocesses to: text 2 (the output cache never marks text
        # valid), first half of image 0, second half 2 (:268-292)
        "final_expected": [2] * txt + [0] * half + [2] * (img - half),
    }
    # --- layer_norm_modulated without gamma/beta (test_gather_scatter.cpp:106-133) ---
    cases["layer_norm"] = {
        "seq_len": 2,
        "dim": 4,
        "eps": 1e-6,
        "x": [1, 2, 3, 4, 5, 6, 7, 8],
        # both rows have variance 1.25 about their mean, so both normalise to the same values
        "expected_row": [-1.3416407, -0.4472136, 0.4472136, 1.3416407],
        "tol": 1e-4,
    }
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(cases, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
