"""Tao history geometry and routing budget (field-for-field the reference ``TaoConfig``).

Reference: tao_attention/config.py:7-63 and tao_attention/presets.py:5-12.  The
fields, their defaults, the validation errors and ``export()`` are kept identical
so that snapshot dictionaries (``StreamCache.export()["config"]``) round-trip
between the reference and this package.
"""

from dataclasses import asdict, dataclass
from math import isqrt

WRITERS = ("softmax", "regularized_association", "feature_mass_association",
           "structured_gram_association")


@dataclass(frozen=True)
class TaoConfig:
    fine_tokens: int = 256
    local_keep: int = 512
    coarse_group: int = 8
    route_period: int = 24
    layer_stagger: int = 2
    budget_root_scale: int = 2
    budget_offset: int = 2
    fine_writer: str = "softmax"
    coarse_index_only: bool = False
    q1_page_normalization_memo: bool = False
    q1_history_region_graph: bool = False

    def __post_init__(self):
        # Same checks and messages as config.py:21-36.
        if self.fine_writer not in WRITERS:
            raise ValueError("unsupported fine writer")
        ints = (self.fine_tokens, self.local_keep, self.coarse_group,
                self.route_period, self.layer_stagger,
                self.budget_root_scale, self.budget_offset)
        if not all(type(v) is int for v in ints):
            raise TypeError("Tao geometry and budget fields must be integers")
        if self.fine_tokens <= 0 or self.local_keep <= 0:
            raise ValueError("fine_tokens and local_keep must be positive")
        if self.local_keep % self.fine_tokens:
            raise ValueError("local_keep must be a multiple of fine_tokens")
        if self.coarse_group <= 0 or self.route_period <= 0:
            raise ValueError("coarse_group and route_period must be positive")
        if self.layer_stagger < 0 or self.budget_root_scale <= 0 or self.budget_offset < 0:
            raise ValueError("unsupported stagger or budget policy")

    @property
    def serve_limit(self):
        """Largest exact local span: ``local_keep + fine_tokens`` (768 in the preset)."""
        return self.local_keep + self.fine_tokens

    @property
    def first_fine(self):
        """First absolute position whose query can read a sealed fine block."""
        return self.serve_limit

    @property
    def first_coarse(self):
        return self.local_keep + self.coarse_group * self.fine_tokens

    @property
    def visibility_tiles(self):
        return self.local_keep // self.fine_tokens

    def budget(self, count):
        """``min(count, ceil(sqrt(root_scale * count)) + offset)``, 0 for empty history."""
        if count <= 0:
            return 0
        square = self.budget_root_scale * count
        root = isqrt(square)
        if root * root < square:
            root += 1
        return min(count, root + self.budget_offset)

    def export(self):
        return asdict(self)


def routed_counts(completed_pages, pending_fine, config):
    """(pages kept by the page top-K, eligible fine candidates, selected fines M).

    Reference: tao_attention/tao_stream.py:29-37.  Pure integer arithmetic; the
    CUDA route kernel evaluates the same formula on the device.
    """
    group = config.coarse_group
    coarse_budget = config.budget(group * completed_pages)
    coarse = min(completed_pages, (2 * coarse_budget + group - 1) // group)
    visible = group * completed_pages + pending_fine
    eligible = group * coarse + pending_fine
    return coarse, eligible, min(eligible, config.budget(visible))


def index_only_page_memo(*, graph=False):
    """The recommended operating preset (reference presets.py:5-12)."""
    return TaoConfig(coarse_index_only=True, q1_page_normalization_memo=True,
                     q1_history_region_graph=graph)
