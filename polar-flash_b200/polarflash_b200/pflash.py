""".pflash container: reader and writer of the reference's on-disk format.

Layout (polarflash_core/formats/pflash_format.py:71-157): b"PFLA", then little-
endian u32 version (1), u32 page alignment, u32 header length; a UTF-8 JSON
header {"metadata": ..., "tensors": [{name, size, shape, dtype, quant_meta,
crc32, offset}]}; payloads at page-aligned absolute offsets.  The reader
validates magic, version, alignment, header bounds and payload bounds and can
check each payload's CRC32 (pflash_format.py:166-259), raising ValueError /
KeyError / RuntimeError as the reference does.
"""
import json
import mmap
import os
import struct
import zlib
from typing import Any, Dict, List, Optional

MAGIC = b"PFLA"
VERSION = 1
DEFAULT_PAGE_ALIGNMENT = 4096


class PFlashWriter:
    def __init__(self, page_alignment: int = DEFAULT_PAGE_ALIGNMENT):
        if page_alignment <= 0 or page_alignment & (page_alignment - 1):
            raise ValueError(f"page_alignment must be a power of 2, got {page_alignment}")
        self.alignment = page_alignment
        self.tensors: List[Dict[str, Any]] = []
        self._names = set()
        self.metadata: Dict[str, Any] = {}

    def set_metadata(self, meta: Dict[str, Any]) -> None:
        self.metadata = meta

    def add_tensor(self, name: str, data_bytes: bytes, shape: List[int], dtype: str,
                   quant_meta: Optional[Dict[str, Any]] = None) -> None:
        if not name or not isinstance(name, str):
            raise ValueError("Tensor name must be a non-empty string.")
        if name in self._names:
            raise ValueError(f"Duplicate tensor name '{name}' registered in .pflash archive.")
        data = bytes(data_bytes)
        self._names.add(name)
        self.tensors.append({"name": name, "bytes": data, "size": len(data), "shape": list(shape),
                             "dtype": dtype, "quant_meta": quant_meta or {}, "crc32": zlib.crc32(data)})

    def _align(self, n: int) -> int:
        return (n + self.alignment - 1) // self.alignment * self.alignment

    def save(self, filepath: str) -> Dict[str, Any]:
        os.makedirs(os.path.dirname(os.path.abspath(filepath)), exist_ok=True)
        catalog = [{k: t[k] for k in ("name", "size", "shape", "dtype", "quant_meta", "crc32")}
                   for t in self.tensors]
        # offsets depend on the header length, which depends on the offsets:
        # iterate until the aligned data start is stable
        data_start = self._align(16)
        while True:
            off = data_start
            for e in catalog:
                e["offset"] = off
                off = self._align(off + e["size"])
            header = json.dumps({"metadata": self.metadata, "tensors": catalog}).encode("utf-8")
            need = self._align(16 + len(header))
            if need <= data_start:
                break
            data_start = need
        with open(filepath, "wb") as f:
            f.write(MAGIC)
            f.write(struct.pack("<III", VERSION, self.alignment, len(header)))
            f.write(header)
            f.write(b"\x00" * (data_start - 16 - len(header)))
            for e, t in zip(catalog, self.tensors):
                assert f.tell() == e["offset"]
                f.write(t["bytes"])
                f.write(b"\x00" * (self._align(f.tell()) - f.tell()))
        size = os.path.getsize(filepath)
        total = self.metadata.get("total_params", sum(_prod(e["shape"]) for e in catalog))
        return {"filepath": filepath, "total_bytes": size, "num_tensors": len(catalog), "total_params": total,
                "effective_bpw": 8.0 * size / max(total, 1), "page_alignment": self.alignment}


def _prod(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


class PFlashReader:
    def __init__(self, filepath: str):
        self.filepath = filepath
        if not os.path.exists(filepath):
            raise FileNotFoundError(f"Archive not found: {filepath}")
        size = os.path.getsize(filepath)
        if size < 16:
            raise ValueError(f"Truncated .pflash file: size is {size} bytes (minimum is 16 bytes).")
        self.file_size = size
        self._closed = True
        self.file_obj = open(filepath, "rb")
        self.mm = mmap.mmap(self.file_obj.fileno(), 0, access=mmap.ACCESS_READ)
        self._closed = False
        try:
            if self.mm[0:4] != MAGIC:
                raise ValueError(f"Invalid .pflash magic bytes: {bytes(self.mm[0:4])}")
            version, alignment, hlen = struct.unpack("<III", self.mm[4:16])
            if version != VERSION:
                raise ValueError(f"Unsupported .pflash format version: {version} (expected {VERSION})")
            if alignment <= 0 or alignment & (alignment - 1):
                raise ValueError(f"Invalid .pflash page alignment: {alignment} (must be a power of 2)")
            if 16 + hlen > size:
                raise ValueError(f"Corrupted .pflash file: header length ({hlen}) extends beyond file size ({size})")
            try:
                header = json.loads(self.mm[16:16 + hlen].decode("utf-8"))
            except Exception as e:  # noqa: BLE001
                raise ValueError(f"Malformed .pflash header JSON: {e}") from e
        except Exception:
            self.close()
            raise
        self.version, self.alignment = version, alignment
        self.metadata = header.get("metadata", {})
        self.tensor_catalog: Dict[str, Dict[str, Any]] = {}
        for t in header.get("tensors", []):
            if t["offset"] + t["size"] > size:
                self.close()
                raise ValueError(f"Corrupted .pflash archive: tensor '{t['name']}' payload (offset {t['offset']}, "
                                 f"size {t['size']}) exceeds file boundary ({size})")
            self.tensor_catalog[t["name"]] = t

    @property
    def catalog(self) -> Dict[str, Dict[str, Any]]:
        return self.tensor_catalog

    def _ensure_open(self) -> None:
        if self._closed:
            raise RuntimeError(f"Operation attempted on closed PFlashReader ({self.filepath})")

    def get_tensor_meta(self, name: str) -> Dict[str, Any]:
        self._ensure_open()
        if name not in self.tensor_catalog:
            raise KeyError(f"Tensor '{name}' not found in .pflash archive")
        return self.tensor_catalog[name]

    def get_tensor_view(self, name: str, verify_checksum: bool = True) -> memoryview:
        info = self.get_tensor_meta(name)
        view = memoryview(self.mm)[info["offset"]:info["offset"] + info["size"]]
        if verify_checksum:
            crc = zlib.crc32(view)
            if crc != info["crc32"]:
                raise ValueError(f"CRC32 mismatch for tensor '{name}': expected {info['crc32']}, got {crc}")
        return view

    def get_tensor_bytes(self, name: str, verify_checksum: bool = True) -> bytes:
        return bytes(self.get_tensor_view(name, verify_checksum))

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            try:
                self.mm.close()
            except Exception:  # noqa: BLE001
                pass
            try:
                self.file_obj.close()
            except Exception:  # noqa: BLE001
                pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
