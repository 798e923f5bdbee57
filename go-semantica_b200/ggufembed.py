"""Host mirror of go-semantica's pkg/ggufembed and the top-level semantica API
(tasks, prompts, Matryoshka dimensions, Runtime.EmbedInputs).

The reference tokenises on the host (internal/tokenizer, kept out of the device
path); Runtime takes the host's `encode(text) -> token ids` callable and sends
every prompt of a request to the device in one batched call.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Iterable, Iterator, Sequence

import numpy as np

# ---- tasks (pkg/ggufembed/tasks.go:12-36) ----
TaskNone = -1
TaskSearchQuery = 0
TaskSearchDocument = 1
TaskQuestionAnswering = 2
TaskFactVerification = 3
TaskClassification = 4
TaskClustering = 5
TaskSemanticSimilarity = 6
TaskCodeRetrieval = 7

_TASK_NAMES = {TaskNone: "none", TaskSearchQuery: "search_query", TaskSearchDocument: "search_document",
               TaskQuestionAnswering: "question_answering", TaskFactVerification: "fact_verification",
               TaskClassification: "classification", TaskClustering: "clustering",
               TaskSemanticSimilarity: "semantic_similarity", TaskCodeRetrieval: "code_retrieval"}

# tasks.go:149-157
DEFAULT_TASK_DESCRIPTIONS = {
    TaskSearchQuery: "search result",
    TaskQuestionAnswering: "question answering",
    TaskFactVerification: "fact checking",
    TaskClassification: "classification",
    TaskClustering: "clustering",
    TaskSemanticSimilarity: "sentence similarity",
    TaskCodeRetrieval: "code retrieval",
}

# tasks.go:84-116 and api.go:26-36
DefaultEmbedDim = 512
Dimensions768, Dimensions512, Dimensions256, Dimensions128 = 768, 512, 256, 128
DimensionsAuto = 0
_SUPPORTED_DIMS = [768, 512, 256, 128]


def task_string(t: int) -> str:
    return _TASK_NAMES.get(t, f"task({t})")


@dataclass
class EmbedInput:
    """pkg/ggufembed/tasks.go:65-82"""
    Task: int = TaskSearchQuery
    Content: str = ""
    Title: str = ""
    CustomTaskDescription: str = ""
    Dim: int = 0


def resolve_dim(dim: int) -> int:
    """ResolveDim (tasks.go:101-109)."""
    if dim == 0:
        return DefaultEmbedDim
    if dim not in _SUPPORTED_DIMS:
        raise ValueError(f"unsupported embed dim {dim} (allowed: 768, 512, 256, 128)")
    return dim


def supported_dims() -> list[int]:
    return list(_SUPPORTED_DIMS)


def build_prompt(inp: EmbedInput) -> str:
    """prompt() (tasks.go:119-147)."""
    content = inp.Content.strip()
    if content == "":
        raise ValueError("content must not be empty")
    if inp.Task == TaskNone:
        return content
    if inp.Task == TaskSearchDocument:
        title = inp.Title.strip() or "none"
        return f"title: {title} | text: {content}"
    desc = inp.CustomTaskDescription.strip()
    if desc == "":
        if inp.Task not in DEFAULT_TASK_DESCRIPTIONS:
            raise ValueError(f"unsupported task {task_string(inp.Task)} (missing default description)")
        desc = DEFAULT_TASK_DESCRIPTIONS[inp.Task]
    return f"task: {desc} | query: {content}"


class Runtime:
    """pkg/ggufembed.Runtime (api.go:14-36) over a device model."""

    def __init__(self, model, encode: Callable[[str], Sequence[int]]):
        self.model = model
        self.encode = encode

    def embed_dim(self) -> int:
        return self.model.config().embed_dim

    def max_seq_len(self) -> int:
        return self.model.config().max_seq_len

    def embed_inputs(self, inputs: Sequence[EmbedInput]) -> list[np.ndarray]:
        """EmbedInputs (api.go:168-187) → one batched forward for every prompt."""
        if len(inputs) == 0:
            return []
        ids, offsets, dims = self._request(inputs)
        return self.model.forward_batch(ids, offsets, dims)

    def _request(self, inputs: Sequence[EmbedInput]):
        ids, offsets, dims = [], [0], []
        for i, inp in enumerate(inputs):
            try:
                prompt = build_prompt(inp)
            except ValueError as e:
                raise ValueError(f"build prompt for input {i}: {e}") from None
            try:
                dim = resolve_dim(inp.Dim)
            except ValueError as e:
                raise ValueError(f"input {i}: {e}") from None
            toks = list(self.encode(prompt))
            if len(toks) > self.max_seq_len():
                raise ValueError(f"sequence too long: {len(toks)} > {self.max_seq_len()}")
            ids.extend(toks)
            offsets.append(len(ids))
            dims.append(dim)
        return np.asarray(ids, dtype=np.int32), np.asarray(offsets, dtype=np.int32), dims

    def embed_inputs_stream(self, batches: Iterable[Sequence[EmbedInput]]) -> Iterator[list[np.ndarray]]:
        """EmbedInputs over a stream of batches through the request pipeline
        (Model.embed_stream): batch i + 1 is tokenised and submitted while the
        device embeds batch i. Yields each batch's vectors in order; empty
        batches yield []."""
        def requests():
            for inputs in batches:
                yield self._request(inputs)
        yield from self.model.embed_stream(requests())

    def embed(self, texts: Sequence[str], task: int = TaskSearchQuery, dim: int = DimensionsAuto) -> list[np.ndarray]:
        """semantica.Runtime.Embed (api.go:90-107)."""
        if len(texts) == 0:
            return []
        d = resolve_dim(dim)
        return self.embed_inputs([EmbedInput(Task=task, Content=t, Dim=d) for t in texts])

    def embed_single(self, text: str, task: int = TaskSearchQuery, dim: int = DimensionsAuto) -> np.ndarray:
        res = self.embed([text], task, dim)
        if not res:
            raise RuntimeError("embed: runtime returned no embeddings")
        return res[0]

    def embed_single_input(self, inp: EmbedInput) -> np.ndarray:
        return self.embed_inputs([inp])[0]
