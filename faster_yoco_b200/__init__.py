"""faster_yoco_b200: a YOCO (You Only Cache Once) pretraining framework written for NVIDIA B200 (sm_100a).

Layers: ``models`` (YOCO decoder-decoder, LLaMA baseline), ``ops`` (op API over the sm_100a kernels in ``csrc``),
``parallel`` (ZeRO-1/2 owner partition, NVLink peer-memory collectives), ``train`` (no-sync trainer, Adam, schedule,
checkpoints), ``data`` (packed LM loader, tokenizers), ``eval`` (harness, needle retrieval, chunked prefill + decode),
``cli`` (fairseq-style train / validate entry points).
"""
__version__ = "0.1.0"
