"""Stand-in base class so diffspec.proposer imports (never instantiated)."""


class AscendEagleProposer:  # pragma: no cover - import shim
    def prepare_next_token_ids_padded(self, *args, **kwargs):
        raise NotImplementedError
