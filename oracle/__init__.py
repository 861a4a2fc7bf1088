"""CPU oracle of the FP8 decoder-layer path (test infrastructure only; see fp8_decoder.py)."""
