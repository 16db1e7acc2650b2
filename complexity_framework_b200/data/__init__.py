"""Data library: token shards (native memory-mapped reader), batch loaders,
packing, tokenizers, chat templates, streaming datasets and mixtures."""
from .loader import (BackgroundTokenizer, CUDAPrefetcher, DataConfig, DistributedDataLoader, InfiniteDataLoader,
                     SyntheticTokenDataset, TokenBatchLoader, create_dataloader)
from .packing import (PackedSequenceCollator, document_attention_mask, pack_documents,
                      packed_labels_and_positions, packing_efficiency)
from .streaming import (CachedDataset, InterleavedDataset, ShardedDataset, StreamingDataset,
                        TokenShardMixture, iter_texts)
from .token_shards import (TokenShardDataset, load_token_shard, open_shard_reader,
                           read_token_shard_metadata, token_shard_frequencies, write_token_shard)
from .tokenization import (IGNORE_INDEX, ByteTokenizer, ChatTemplate, HuggingFaceTokenizer, Message,
                           SentencePieceTokenizer, TiktokenWrapper, Tokenizer, ToolDefinition,
                           encode_chat, get_tokenizer)
