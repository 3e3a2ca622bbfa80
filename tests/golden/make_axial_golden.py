"""Writes axial_reference.json: the known answers of the reference's own
oracle tests, transcribed from Tests/H3AttentionTests/AxialReferenceTests.swift
(MiniMax-H3-Swift).  The reference cannot run here (Swift/MLX on macOS), so
its literal expectations are the pin for the mask semantics.

  fixture            :22-34   prefix 7, frames 5, 3x4 lattice, landmarks [0, 4]
  spot checks        :119-143 token 37 -> (frame 2, y 1, x 2); allowed keys
                              3, 31, 61, 12, 60; excluded key 19
  density            :145-160 counted == closed form (prefix 7, frames 6)
  geometry refusal   :162-174 864x480x124: video 746..<15731 ok, 700.. / ..15000 refused
  landmarks          :176-193 37 frames: [0, 18, 36]; landmarks 1 -> [0, 36]; 999 -> all 37
  LatentGeometry     Sources/H3Foundation/LatentGeometry.swift:29-37 with
                     H3Config.swift:74-84: latentT 37, latentH 30, latentW 54
"""
import json
import os

GOLDEN = {
    "fixture": {"prefix": 7, "frames": 5, "height": 3, "width": 4, "landmarks": [0, 4]},
    "spot": {"query": 37, "locate": [2, 1, 2], "allowed": [3, 31, 61, 12, 60], "excluded": [19]},
    "density_fixture": {"prefix": 7, "frames": 6, "height": 3, "width": 4, "landmarks": [0, 5]},
    "geometry": {"width": 864, "height": 480, "length": 124, "latent_t": 37, "latent_h": 30, "latent_w": 54,
                 "seq_len": 15731, "video_ok": [746, 15731], "video_bad": [[700, 15731], [746, 15000]]},
    "landmarks": {"3": [0, 18, 36], "1": [0, 36], "999_count": 37},
}

if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "axial_reference.json")
    with open(out, "w") as f:
        json.dump(GOLDEN, f, indent=1)
    print(out)
