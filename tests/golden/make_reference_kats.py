"""Write tests/golden/reference_kats.json.

The vectors are the literal inputs and asserted outputs of the reference's own
unit tests (MangoByteLabs/vortex), transcribed by hand with their file:line:
  int4 pack:   src/quantize.rs:928-935 ([0,1,-1,7,-8,3,-4,5]; low nibble = even index)
  Q4_0 block:  src/gguf_loader.rs:857-878 (d=0x3C00, byte0=0xA9, rest 0x88 -> [1,2,0,...])
  Q8_0 block:  src/gguf_loader.rs:881-895 (d=0x3C00, bytes 3, 0xFD -> [3,-3,0,...])
  f16 decode:  src/gguf_loader.rs:932-940 (0x3C00, 0xBC00, 0x3800 -> 1, -1, 0.5)
Run: python tests/golden/make_reference_kats.py
"""
import json
import os


def main():
    q4 = [0x00, 0x3C, 0xA9] + [0x88] * 15
    q8 = [0x00, 0x3C, 3, 0xFD] + [0] * 30
    kats = {
        "source": "MangoByteLabs/vortex unit tests (see make_reference_kats.py)",
        "int4_pack": [{"values": [0, 1, -1, 7, -8, 3, -4, 5], "packed": [0x10, 0x7F, 0x38, 0x5C]}],
        "q4_0_block": [{"block": q4, "values": [1.0, 2.0] + [0.0] * 30}],
        "q8_0_block": [{"block": q8, "values": [3.0, -3.0] + [0.0] * 30}],
        "f16": [{"bits": 0x3C00, "value": 1.0}, {"bits": 0xBC00, "value": -1.0},
                {"bits": 0x3800, "value": 0.5}],
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(path, "w") as f:
        json.dump(kats, f, indent=1)


if __name__ == "__main__":
    main()
