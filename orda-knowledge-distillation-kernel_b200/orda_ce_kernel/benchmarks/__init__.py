"""Benchmarks that a user of the library runs on a B200 (``python -m orda_ce_kernel.benchmarks.<name>``):
``accuracy`` (loss / gradient error against an fp32 PyTorch formula), ``vram`` (peak extra device
memory of one loss + backward) and ``train_step`` (a small Transformer student trained with the loss)."""
