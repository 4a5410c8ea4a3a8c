"""Images in OpenAI-style chat messages -> PIL images plus messages whose image parts became
the vision model's placeholder text.

Accepted parts: ``{"type": "image_url", "image_url": {"url": ...}}`` (or ``"image_url": "..."``)
and ``{"type": "image", "image": ...}``, where the value is a ``data:image/...;base64,`` URL, bare
base64, or the id of a file uploaded to ``/v1/files``. Remote http(s) URLs are refused (the
server fetches nothing on a client's behalf). Content lists are flattened to text with each image
replaced by ``<|vision_start|><|image_pad|><|vision_end|>``, which the engine expands to the
image's visual tokens. Reference behaviour: core/engine_transformers.py:1134-1189 (images taken
from the messages and handed to the processor).
"""

from __future__ import annotations

import base64
import binascii
import io
from typing import List, Tuple

PLACEHOLDER = "<|vision_start|><|image_pad|><|vision_end|>"
MAX_IMAGE_BYTES = 32 << 20


class ImageError(ValueError):
    pass


def _decode(value: str, files=None):
    from PIL import Image
    if not isinstance(value, str) or not value:
        raise ImageError("image value must be a data URL, base64 or a file id")
    if value.startswith(("http://", "https://")):
        raise ImageError("remote image URLs are not fetched; upload the image to /v1/files or send a data URL")
    if value.startswith("file-"):
        from b200serve.core.file_store import get_file_store
        store = files or get_file_store()
        data = store.read(value)
        if data is None:
            raise ImageError(f"no such file: {value}")
    else:
        b64 = value.split(",", 1)[1] if value.startswith("data:") else value
        try:
            data = base64.b64decode(b64, validate=False)
        except (binascii.Error, ValueError) as e:
            raise ImageError(f"image is not valid base64: {e}")
    if len(data) > MAX_IMAGE_BYTES:
        raise ImageError(f"image larger than {MAX_IMAGE_BYTES >> 20} MB")
    try:
        img = Image.open(io.BytesIO(data))
        img.load()
    except Exception as e:                     # PIL raises several exception types on bad input
        raise ImageError(f"cannot decode image: {e}")
    return img


def extract_images(messages: List[dict], files=None) -> Tuple[List[dict], list]:
    """(messages with text content only, images in order of appearance)."""
    images, out = [], []
    for m in messages:
        c = m.get("content")
        if not isinstance(c, list):
            out.append(m)
            continue
        text = []
        for part in c:
            if not isinstance(part, dict):
                continue
            kind = part.get("type")
            if kind == "text":
                text.append(part.get("text", ""))
            elif kind in ("image_url", "image"):
                v = part.get("image_url") if kind == "image_url" else part.get("image")
                if isinstance(v, dict):
                    v = v.get("url")
                images.append(_decode(v, files))
                text.append(PLACEHOLDER)
        out.append(dict(m, content="".join(text)))
    return out, images
