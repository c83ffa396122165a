"""Persistent KV-record ABI of packmla (byte layouts shared by every kernel).

C4 records (one record = the compressed latent of 4 consecutive tokens) come in
two layouts, matching the reference's formats (docs/report.md:9,
docs/agents/numerical-and-validation.md:10-16, training/tests/test_integration.py:361-364):

Native record, 584 logical bytes
    data row (576 B): [0, 448)   448 E4M3 NoPE coordinates
                      [448, 576) 64 BF16 RoPE coordinates, already rotated
    scale row (8 B):  7 UE8M0 codes (one per 64-coordinate NoPE tile) + 1 pad byte (0)

    Pages hold RECORDS_PER_PAGE records: all data rows first, then all scale rows,
    so every data row starts on a 16-byte boundary (576 = 36 * 16).

Packed record, 328 logical bytes, three planes indexed by physical record id
    values plane  uint8[rows, 256]   E4M3 survivors in ascending coordinate order
    bitmap plane  uint64[rows, 8]    word w covers coordinates [64w, 64w+64);
                                     bit b (LSB = 0) marks coordinate 64w + b as kept
    scale plane   uint8[rows, 8]     UE8M0 code per 64-coordinate tile (RoPE tile included)

    Packed values are pre-RoPE; readers rotate the tail with the record's position.

The bitmap bit order is not stated by the reference for the FP8 V4 layout; packmla
fixes LSB-first words here and tests it.
"""

LATENT_DIM = 512
NOPE_DIM = 448
ROPE_DIM = 64
ROPE_PAIRS = ROPE_DIM // 2
TILE = 64
NUM_TILES = LATENT_DIM // TILE  # 8
NOPE_TILES = NOPE_DIM // TILE  # 7

E4M3_MAX = 448.0
UE8M0_BIAS = 127
AMAX_FLOOR = 1e-4

NATIVE_DATA_BYTES = NOPE_DIM + ROPE_DIM * 2  # 576
NATIVE_SCALE_BYTES = 8
NATIVE_RECORD_BYTES = NATIVE_DATA_BYTES + NATIVE_SCALE_BYTES  # 584

PACKED_KEEP = 256
BITMAP_WORDS = LATENT_DIM // 64  # 8
PACKED_BITMAP_BYTES = BITMAP_WORDS * 8  # 64
PACKED_SCALE_BYTES = NUM_TILES  # 8
PACKED_RECORD_BYTES = PACKED_KEEP + PACKED_BITMAP_BYTES + PACKED_SCALE_BYTES  # 328

RECORDS_PER_PAGE = 64  # one page = 256 tokens = 64 C4 records
NATIVE_PAGE_BYTES = RECORDS_PER_PAGE * NATIVE_RECORD_BYTES  # 37376 (16-byte multiple)

C4_RATIO = 4
C128_RATIO = 128
SWA_WINDOW = 128

RETENTION_COUNTS = tuple(range(64, 449, 64))


def packed_record_bytes(keep: int) -> int:
    """Logical bytes of a Packed record keeping `keep` of 512 coordinates (K + 72)."""
    if keep not in RETENTION_COUNTS:
        raise ValueError(f"keep count {keep} not in {RETENTION_COUNTS}")
    return keep + PACKED_BITMAP_BYTES + PACKED_SCALE_BYTES


def native_slot_offsets(slot: int) -> tuple[int, int]:
    """(data byte offset, scale byte offset) of a Native record in the paged pool."""
    page, r = divmod(slot, RECORDS_PER_PAGE)
    base = page * NATIVE_PAGE_BYTES
    return base + r * NATIVE_DATA_BYTES, base + RECORDS_PER_PAGE * NATIVE_DATA_BYTES + r * NATIVE_SCALE_BYTES
