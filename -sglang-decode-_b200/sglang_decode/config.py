"""Capture-time capacities and immutable attention geometry.

Mirrors the reference's ``config.py:1-58`` (field names, defaults semantics, derived
properties).  Differences, by design of the B200 build:

* any integer GQA group 1..16 is accepted (e.g. Qwen2-7B's 7), not only powers of two;
* ``workers`` defaults to 148, the B200 SM count (one persistent CTA per SM).
"""
from dataclasses import dataclass
from enum import IntEnum


class Mode(IntEnum):
    R0 = 0  # compact prefix-search round robin
    R1 = 1  # direct-record round robin
    STATIC = 2  # longest-processing-time greedy lists
    D1 = 3  # one logical task per atomic claim
    D4 = 4  # bounded short-task packs


SUPPORTED_HEAD_DIMS = (64, 128, 256)
MAX_GROUP = 16
MAX_RECORDS = 4096


@dataclass(frozen=True)
class DecodeConfig:
    batch_capacity: int = 64
    max_splits: int = 16
    max_context: int = 32768
    query_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    page_size: int = 16
    workers: int = 148
    block_kv: int = 128
    split_alignment: int = 32

    def __post_init__(self):
        for name, value in vars(self).items():
            if value <= 0:
                raise ValueError(f"{name} must be positive")
        if self.query_heads % self.kv_heads or not 1 <= self.group_size <= MAX_GROUP:
            raise ValueError("query heads must be a multiple 1..16 of KV heads")
        if self.head_dim not in SUPPORTED_HEAD_DIMS:
            raise ValueError("supported head dimensions: 64, 128, 256")
        if self.block_kv != 128 or self.split_alignment != 32:
            raise ValueError("this kernel specialization uses tile=128 and split alignment=32")
        if self.record_capacity > MAX_RECORDS or self.task_capacity >= 2**31:
            raise ValueError("planner bound exceeded; choose another instance or upstream")
        if self.workers > 4096:
            raise ValueError("at most 4096 persistent workers")

    @property
    def group_size(self):
        return self.query_heads // self.kv_heads

    @property
    def record_capacity(self):
        return self.batch_capacity * self.max_splits

    @property
    def task_capacity(self):
        return self.record_capacity * self.kv_heads

    @property
    def max_pages(self):
        return (self.max_context + self.page_size - 1) // self.page_size

    @property
    def buckets(self):
        return ((self.max_context + self.block_kv - 1) // self.block_kv - 1).bit_length() + 1
