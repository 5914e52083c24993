"""Golden vectors for the input preprocessing of the reference's classification
demo (demo/image_classification.cpp:9-44), produced with OpenCV itself:

    cv::resize(image, image, cv::Size(256, 256));          // INTER_LINEAR
    cv::cvtColor(image, image, cv::COLOR_BGR2RGB);
    image.convertTo(image, CV_32FC3, 1.f / 255.f);
    crop 224 x 224 at (max(0, cx - 112), max(0, cy - 112));
    per channel (x - mean[c]) / stddev[c], planar [3][224][224]

The reference builds against whatever OpenCV find_package() finds (no version
pin); these vectors come from the cv2 module of the build container (its
version is stored in the file).  Inputs are seeded random 8-bit BGR images,
one downscaled and one upscaled.

    python tests/golden/make_preprocess_golden.py    -> tests/golden/preprocess_cv2.npz
"""
import os

import cv2
import numpy as np

MEAN = (0.485, 0.456, 0.406)
STD = (0.229, 0.224, 0.225)


def reference_preprocess(img_bgr: np.ndarray) -> np.ndarray:
    image = cv2.resize(img_bgr, (256, 256))
    image = cv2.cvtColor(image, cv2.COLOR_BGR2RGB)
    image = image.astype(np.float32) * np.float32(1.0 / 255.0)
    cx, cy = image.shape[1] // 2, image.shape[0] // 2
    x, y = max(0, cx - 112), max(0, cy - 112)
    crop = image[y:y + 224, x:x + 224]
    out = np.empty((3, 224, 224), np.float32)
    for c in range(3):
        out[c] = (crop[:, :, c] - MEAN[c]) / STD[c]
    return out


def main():
    rng = np.random.default_rng(2024)
    images = {"down_320x240": rng.integers(0, 256, (240, 320, 3), dtype=np.uint8),
              "up_150x200": rng.integers(0, 256, (150, 200, 3), dtype=np.uint8)}
    arrays = {"cv2_version": np.array(cv2.__version__)}
    for name, img in images.items():
        arrays[name + "_bgr"] = img
        arrays[name + "_out"] = reference_preprocess(img)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "preprocess_cv2.npz")
    np.savez_compressed(path, **arrays)
    print(path, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
