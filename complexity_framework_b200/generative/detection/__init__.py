"""TR-Hash object detection (counterpart: complexity/generative/detection/)."""
from .augmentations import (AugmentedDataset, DetectionAugment, color_jitter, horizontal_flip,
                            mosaic, random_scale)
from .coco_evaluation import evaluate_detections
from .config import COCO_V8_NANO_NAME, TRHashDetectorConfig, coco_v8_nano_config
from .data import (COCO_CLASS_NAMES, VOC_CLASS_NAMES, CocoDetectionDataset,
                   DetectionImageMetadata, SyntheticShapesDataset, YoloDetectionDataset,
                   collate_detection, preprocess_detector_image, restore_detector_boxes)
from .ema import ModelEMA
from .exporting import (export_detector_torchscript, load_detector_checkpoint,
                        save_detector_checkpoint)
from .losses import distribution_focal_loss, quality_focal_loss
from .model import TRHashObjectDetector
from .ops import box_iou, class_aware_nms, complete_iou, complete_iou_loss, greedy_nms
from .trainer import DetectorTrainer, DetectorTrainingConfig
from .metrics import DetectionMetricsAccumulator, evaluate_predictions
from .checkpointing import load_training_state, save_training_state
from .distributed import DistributedContext, DistributedEvalSampler
from .train import DetectorRunConfig, train_detector

__all__ = [
    "TRHashDetectorConfig", "TRHashObjectDetector", "box_iou", "class_aware_nms",
    "complete_iou", "complete_iou_loss", "greedy_nms", "COCO_V8_NANO_NAME", "coco_v8_nano_config",
    "distribution_focal_loss", "quality_focal_loss", "CocoDetectionDataset",
    "SyntheticShapesDataset", "YoloDetectionDataset", "collate_detection", "COCO_CLASS_NAMES",
    "VOC_CLASS_NAMES", "DetectionImageMetadata", "preprocess_detector_image",
    "restore_detector_boxes", "ModelEMA", "evaluate_detections", "save_detector_checkpoint",
    "load_detector_checkpoint", "export_detector_torchscript", "DetectorTrainer",
    "DetectorTrainingConfig", "DetectionAugment", "AugmentedDataset", "mosaic",
    "horizontal_flip", "random_scale", "color_jitter", "DetectionMetricsAccumulator",
    "evaluate_predictions", "save_training_state", "load_training_state", "DistributedContext",
    "DistributedEvalSampler", "DetectorRunConfig", "train_detector",
]
