"""HRM-Text pretraining / SFT entry point (same command line as the reference's pretrain.py).

    OMP_NUM_THREADS=1 torchrun --nproc_per_node=8 pretrain.py arch/size@arch=L lr=2.5e-4 \
        global_batch_size=172032
    torchrun --nproc_per_node=8 pretrain.py --config-name cfg_sft arch/size@arch=XL \
        data.path=/dev/shm/sft_data resume_from=/path/to/pretrain_ckpt +checkpoint_path=/path/to/sft_out
"""
from hrm_text_b200.runtime.pretrain import main

if __name__ == "__main__":
    main()
