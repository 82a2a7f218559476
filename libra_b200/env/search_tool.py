"""Web/corpus search tool for the Search-R1 workflow.

Role of the reference's ``env/search_tool.py:19-158`` (Serper or SearXNG
backends, numbered result formatting).  Adds an offline ``local`` backend: BM25
over a JSONL corpus of ``{"title", "text"[, "url"]}`` documents, for boxes
without network access and for tests.
"""

from __future__ import annotations

import asyncio
import json
import math
import os
import re
from collections import Counter
from typing import Dict, List, Optional

_TOKEN = re.compile(r"\w+", re.UNICODE)


def _has_cjk(text: str) -> bool:
    return any("一" <= ch <= "鿿" for ch in text)


def format_results(query: str, pages: List[Dict], max_results: int) -> str:
    items = []
    for i, p in enumerate(pages[:max_results], 1):
        date = p.get("publishedDate") or p.get("date") or ""
        items.append(f"{i}. [{p.get('title', '')}]({p.get('url') or p.get('link', '')})"
                     + (f"\nDate: {date}" if date else "") + f"\n{p.get('content') or p.get('snippet', '')}")
    if not items:
        return f"No results found for query: '{query}'. Try a more general query."
    return f"Search results for '{query}' ({len(items)} results):\n\n" + "\n\n".join(items)


class BM25Corpus:
    def __init__(self, docs: List[Dict], k1: float = 1.5, b: float = 0.75):
        self.docs, self.k1, self.b = docs, k1, b
        self.tf = [Counter(_TOKEN.findall((d.get("title", "") + " " + d.get("text", "")).lower())) for d in docs]
        self.len = [sum(c.values()) for c in self.tf]
        self.avg = sum(self.len) / max(len(self.len), 1)
        df = Counter(w for c in self.tf for w in c)
        n = len(docs)
        self.idf = {w: math.log(1 + (n - f + 0.5) / (f + 0.5)) for w, f in df.items()}

    @classmethod
    def from_jsonl(cls, path: str) -> "BM25Corpus":
        with open(path, encoding="utf-8") as f:
            return cls([json.loads(line) for line in f if line.strip()])

    def search(self, query: str, k: int) -> List[Dict]:
        q = _TOKEN.findall(query.lower())
        scores = []
        for i, tf in enumerate(self.tf):
            s = 0.0
            for w in q:
                if w in tf:
                    f = tf[w]
                    s += self.idf[w] * f * (self.k1 + 1) / (f + self.k1 * (1 - self.b + self.b * self.len[i] / self.avg))
            if s > 0:
                scores.append((s, i))
        scores.sort(reverse=True)
        return [{"title": self.docs[i].get("title", ""), "url": self.docs[i].get("url", ""),
                 "snippet": self.docs[i].get("text", "")[:500]} for _, i in scores[:k]]


class SearchTool:
    def __init__(self, api_key: Optional[str] = None, max_results: int = 5, backend: Optional[str] = None,
                 searxng_url: Optional[str] = None, corpus: Optional[BM25Corpus] = None, timeout_s: float = 20.0,
                 retries: int = 2):
        self.api_key = api_key or os.environ.get("SERPER_KEY_ID", "")
        self.max_results = max_results
        self.backend = (backend or os.environ.get("SEARCH_BACKEND", "local" if corpus else "serper")).lower()
        if self.backend not in ("serper", "searxng", "local"):
            raise ValueError(f"unsupported search backend {self.backend!r} (serper, searxng or local)")
        self.searxng_url = (searxng_url or os.environ.get("SEARXNG_URL", "http://127.0.0.1:8080")).rstrip("/")
        if self.backend == "local" and corpus is None and os.environ.get("SEARCH_CORPUS_JSONL"):
            corpus = BM25Corpus.from_jsonl(os.environ["SEARCH_CORPUS_JSONL"])
        self.corpus = corpus
        self.timeout_s, self.retries = timeout_s, retries

    async def _http(self, method: str, url: str, **kw) -> Dict:
        import aiohttp

        last = None
        for attempt in range(self.retries + 1):
            try:
                async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=self.timeout_s)) as s:
                    async with s.request(method, url, **kw) as r:
                        r.raise_for_status()
                        return await r.json(content_type=None)
            except Exception as exc:  # noqa: BLE001 - retried, then reported as text
                last = exc
                await asyncio.sleep(0.5 * (attempt + 1))
        raise RuntimeError(str(last))

    async def search(self, query: str) -> str:
        query = (query or "").strip()
        if not query:
            return "[Search Error] empty query."
        try:
            if self.backend == "local":
                if self.corpus is None:
                    return "[Search Error] no local corpus configured."
                pages = self.corpus.search(query, self.max_results)
            elif self.backend == "serper":
                if not self.api_key:
                    return "[Search Error] SERPER_KEY_ID not configured."
                cjk = _has_cjk(query)
                body = await self._http("POST", "https://google.serper.dev/search",
                                        json={"q": query, "gl": "cn" if cjk else "us", "hl": "zh-cn" if cjk else "en"},
                                        headers={"X-API-KEY": self.api_key})
                pages = body.get("organic", [])
            else:
                body = await self._http("GET", f"{self.searxng_url}/search", params={"q": query, "format": "json"})
                pages = body.get("results", [])
        except Exception as exc:  # noqa: BLE001 - the model sees the failure as the tool output
            return f"[Search Error] {exc}"
        return format_results(query, pages, self.max_results)

    async def search_batch(self, queries: List[str]) -> List[str]:
        return list(await asyncio.gather(*(self.search(q) for q in queries)))
