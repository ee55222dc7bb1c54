"""Host-side package of the B200 RF-DETR engine: the ctypes binding of
librfdetr.so (lib) and the seeded synthetic GGUF writer (synth)."""
